"""B200 compositions behind the reference's ``minifield_training.layers`` names."""
