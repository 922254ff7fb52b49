"""B200 (sm_100a) implementation of ds-ocr's MoE-decoder hot path.

The compute lives in libds_cuda.so (hand-written CUDA, C ABI in
include/ds_cuda.h); this package is the Python host side: the ctypes binding
(_lib, cuda), the decoder engine (decoder) and synthetic workloads (synth).
"""
__all__ = ["cuda", "synth", "decoder"]
