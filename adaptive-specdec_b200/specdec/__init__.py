"""B200-native drop-in for the reference specdec package (verify-round hot path)."""
