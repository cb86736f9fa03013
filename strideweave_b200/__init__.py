"""B200-native CUDA carrier for StrideWeave (contraction and reduction hot path)."""
