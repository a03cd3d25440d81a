"""vauss_b200: B200-native Gaussian-splat training step."""
