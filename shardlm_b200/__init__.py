"""shardlm_b200: B200-native (sm_100a) secret-shared transformer forward pass for ShardLM.

The compute path is libshardlm_cuda.so (C ABI in include/shardlm_cuda.h); this package is the
host-side mirror of the reference's layer API on top of it.
"""
__version__ = "0.1.0"
