"""B200-native W4A8 ConvRot quantised linear for the MiniMax H3 DiT (sm_100a kernels behind a C-ABI)."""
__version__ = "0.1.0"
