"""B200 kernels behind the reference's ``minifield_training.kernels`` names."""
