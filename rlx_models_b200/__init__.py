"""rlx_models_b200 - a Blackwell (sm_100a)-native model framework.

PyTorch is the framework layer; the hot paths are this package's own CUDA
kernels (tcgen05/TMEM GEMMs fed by TMA, paged attention, fused norm/RoPE,
on-GPU sampling, fused AdamW) and its NVLink peer-memory collectives.
"""
__version__ = "0.1.0"
