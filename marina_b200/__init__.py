"""marina_b200: a B200-native evaluator for Marina's batched transformer forward."""
