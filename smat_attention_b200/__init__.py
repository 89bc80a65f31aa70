"""SMat block-sparse causal softmax attention for NVIDIA B200 (sm_100a)."""
