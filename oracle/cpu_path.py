"""TEST / BASELINE INFRASTRUCTURE ONLY: the reference's own CPU code path, restated.

The reference (gtx16_fp16) has no CPU kernels. Its CPU behaviour is the torch fallback that every
entry point takes when the inputs are not fp16/fp32 CUDA tensors of a supported shape:

* ``matmul`` -> ``torch.matmul(a, b).to(out_dtype)`` (src/gtx16_fp16/ops.py:119);
* ``FastLinear.forward`` -> ``F.linear(x.float(), w_t.t().float(), bias)`` (src/gtx16_fp16/linear.py:188-189),
  i.e. an fp32 matmul.

bench.py times these on the host cores (all threads) as the CPU baseline and as the ``--impl
reference`` arm; tests compare them with the golden vectors recorded from the reference itself.
"""
from __future__ import annotations

import os

import torch
import torch.nn.functional as F


def use_all_cores() -> int:
    n = os.cpu_count() or 1
    torch.set_num_threads(n)
    return torch.get_num_threads()


def matmul(a: torch.Tensor, b: torch.Tensor, out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """ops.py:111-119 on CPU tensors: torch's matmul in the input dtype, then cast."""
    out_dtype = out_dtype or torch.float16
    return torch.matmul(a, b).to(out_dtype)


def mm_t_fp32(x2d: torch.Tensor, w_t: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
    """The fp32 fallback of linear.py:188-189: out = x.float() @ w_t.float() + bias."""
    return F.linear(x2d.float(), w_t.t().float(), bias)
