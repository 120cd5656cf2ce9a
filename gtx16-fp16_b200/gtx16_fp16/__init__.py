"""B200-native (sm_100a) fp16 matmul with the gtx16_fp16 API.

    import gtx16_fp16
    n = gtx16_fp16.patch(model, force=True)   # swap nn.Linear -> FastLinear
    y = gtx16_fp16.matmul(a16, b16)           # tcgen05 tensor-core GEMM, fp16 out like torch
    y = gtx16_fp16.mm_t(x, w_t, bias, torch.float32)
    step = gtx16_fp16.graphs.capture(fn, x)   # CUDA-graph a decode step (no host cost per layer)

Drop-in for the reference package's surface (src/gtx16_fp16/__init__.py:7-11). The kernels live in
libg16.so (include/g16.h), built in-tree for sm_100a.
"""
from . import graphs
from .linear import FastLinear, patch
from .ops import ROW_SCALE_THRESHOLD, SKINNY_MAX_M, is_affected, matmul, mm_t, skinny_config, supported

__all__ = ["FastLinear", "patch", "is_affected", "matmul", "mm_t", "supported"]
__version__ = "0.1.0"
