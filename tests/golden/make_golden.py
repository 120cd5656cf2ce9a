"""Generate tests/golden/ fixtures by running the reference package itself (build container only).

The reference (gtx16_fp16) is imported from its read-only checkout; only its CPU-runnable code runs
here (no GPU in the build container):
  * ``skinny_config`` (src/gtx16_fp16/ops.py:45-51), pure integer arithmetic;
  * ``matmul`` on CPU tensors -> its torch fallback (ops.py:119), BASELINE config 1 inputs;
  * ``FastLinear`` forward on CPU -> its fp32 ``F.linear`` fallback (linear.py:184-192);
  * ``supported`` / ``is_affected`` / ``patch`` results on CPU, constants and ``__all__``.
Outputs: tests/golden/reference_cpu.npz and tests/golden/reference_meta.json. Inputs are regenerated
from torch's CPU generator with the recorded seeds, so only outputs (and digests) are stored.

Usage: python tests/golden/make_golden.py --reference <reference checkout>
       (or set G16_REFERENCE_DIR; there is no default location)
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def config1_inputs(M=1024, K=1024, N=1024, seed=0):
    """A ~ N(0,1) fp16, B ~ N(0, 1/sqrt(K)) fp16 (std K^-1/2), torch CPU generator."""
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(M, K, generator=g).half()
    b = (torch.randn(K, N, generator=g) * K ** -0.5).half()
    return a, b


def linear_inputs(seed=0):
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(768, 1024, generator=g) * 0.03  # nn.Linear(1024, 768).weight layout [out, in]
    bias = torch.randn(768, generator=g) * 0.1
    x = torch.randn(2, 8, 1024, generator=g)
    return w, bias, x


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().numpy().tobytes()).hexdigest()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("G16_REFERENCE_DIR"),
                    help="reference checkout (default: $G16_REFERENCE_DIR)")
    a = ap.parse_args()
    if not a.reference:
        ap.error("give --reference or set G16_REFERENCE_DIR")
    sys.path.insert(0, os.path.join(a.reference, "src"))
    import gtx16_fp16 as ref  # the reference package
    from gtx16_fp16 import ops as ref_ops

    torch.set_num_threads(1)  # fixed reduction order for the CPU fp16 GEMM
    meta = {"generator": "tests/golden/make_golden.py", "torch": torch.__version__,
            "reference_all": list(ref.__all__), "ROW_SCALE_THRESHOLD": ref_ops.ROW_SCALE_THRESHOLD,
            "SKINNY_MAX_M": __import__("gtx16_fp16.kernels", fromlist=["x"]).SKINNY_MAX_M}
    arrays = {}

    # skinny_config over a grid of shapes and SM counts
    rows = []
    for sms in (24, 132, 148, 160):
        for N in (8, 136, 256, 520, 776, 1024, 3072, 4096, 4104, 16384):
            for K in (8, 64, 136, 520, 1024, 2048, 3072, 4096, 16384):
                grid, kchunk = ref.ops.skinny_config(N, K, sms)
                rows.append([N, K, sms, grid[0], grid[1], grid[2], kchunk])
    arrays["skinny_config"] = np.array(rows, dtype=np.int64)

    # config 1 through the reference's CPU path (matmul fallback), full digest + first rows
    a1, b1 = config1_inputs()
    y1 = ref.matmul(a1, b1)
    meta["config1"] = {"shape": [1024, 1024, 1024], "seed": 0, "dtype": str(y1.dtype), "sha256": sha(y1),
                       "threads": 1}
    arrays["config1_rows0_7"] = y1[:8].numpy()
    a_s, b_s = config1_inputs(32, 64, 48, seed=3)
    arrays["small_matmul"] = ref.matmul(a_s, b_s).numpy()
    arrays["small_matmul_f32"] = ref.matmul(a_s, b_s, out_dtype=torch.float32).numpy()

    # FastLinear on CPU: fp32 F.linear fallback
    w, bias, x = linear_inputs()
    lin = torch.nn.Linear(1024, 768)
    with torch.no_grad():
        lin.weight.copy_(w)
        lin.bias.copy_(bias)
    fl = ref.FastLinear.from_linear(lin)
    with torch.no_grad():
        yl = fl(x)
    arrays["fastlinear_cpu"] = yl.numpy()
    meta["fastlinear_cpu"] = {"dtype": str(yl.dtype), "shape": list(yl.shape),
                              "state_dict_keys": sorted(fl.state_dict().keys()),
                              "weight_t_dtype": str(fl.weight_t.dtype), "bias_dtype": str(fl.bias.dtype),
                              "extra_repr": fl.extra_repr()}

    # host-side decisions on CPU
    meta["supported_cpu"] = bool(ref.supported(a_s, b_s))
    meta["is_affected"] = bool(ref.is_affected())
    model = torch.nn.Sequential(torch.nn.Linear(512, 1024), torch.nn.GELU(), torch.nn.Linear(1024, 512))
    meta["patch_cpu_force"] = ref.patch(model, min_features=256, force=True)
    meta["patch_cpu_noforce"] = ref.patch(model)
    try:
        ref.mm_t(a_s, b_s, None, torch.bfloat16)
        meta["mm_t_bad_dtype"] = None
    except ValueError as e:
        meta["mm_t_bad_dtype"] = str(e)

    np.savez_compressed(os.path.join(HERE, "reference_cpu.npz"), **arrays)
    with open(os.path.join(HERE, "reference_meta.json"), "w") as f:
        json.dump(meta, f, indent=1, sort_keys=True)
    print("wrote", sorted(arrays), "and meta keys", sorted(meta))


if __name__ == "__main__":
    main()
