"""Generate the golden NVFP4 vectors in this directory by running the reference package itself.

    PYTHONPATH=<reference checkout> PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py

The reference (nvfp4_gemm_cute 0.1.0) is imported read-only; its quantize_nvfp4 / swizzle_sf /
dequantize_nvfp4 (quant.py:31-70) run on CPU tensors with this container's torch, and its FP32
reference matmul (testing.py:18-27) gives the GEMM case. Inputs are seeded and synthetic. The
output, golden.npz, is what tests/test_oracle_golden.py and the GPU parity tests compare
against; nothing at test time needs the reference.
"""

import os
import sys

import numpy as np
import torch

from nvfp4_gemm_cute.quant import dequantize_nvfp4, quantize_nvfp4, swizzle_sf  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden.npz")


def ties_block():
    """Rows built around E2M1 rounding ties, signs, zeros, tiny and non-finite values."""
    base = torch.tensor(
        [
            [0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, -0.1, 0.1, 1.2500005, 1.2500015, 6.0, -6.0, 0.0, -0.0, 3.0],
            [-0.25, -0.75, -1.25, -1.75, -2.5, -3.5, -5.0, 0.2499999, 0.2500001, 0.7499999, 0.7500001,
             4.9999995, 5.0000005, 2.4999998, 2.5000002, 6.0],
            [1e-3, 2e-3, -3e-3, 4e-3, 5e-3, 6e-3, 7e-3, 8e-3, 9e-3, 1e-2, -1.1e-2, 1.2e-2, 1.3e-2, 1.4e-2,
             1.5e-2, 1.6e-2],
            [1e-9, -2e-9, 3e-9, 0.0, 0.0, -0.0, 0.0, 0.0, 1e-9, 0.0, 0.0, 0.0, 0.0, 0.0, 0.0, 5e-9],
            [0.0] * 16,
            [-0.0] * 16,
            [460.0 * 6, 1.0, -2.0, 3.0, 4.0, 5.0, 6.0, 7.0, 8.0, 9.0, 10.0, 11.0, 12.0, 13.0, 14.0, 15.0],
            [464.0 * 6, 1.0, -2.0, 3.0, 4.0, 5.0, 6.0, 7.0, 8.0, 9.0, 10.0, 11.0, 12.0, 13.0, 14.0, 15.0],
            [3000.0, -1.0] + [0.5] * 14,
            [float("inf"), 1.0] + [0.25] * 14,
            [float("nan"), 1.0] + [0.25] * 14,
            [7.125 - 4.76837158203125e-07] + [1.0] * 15,  # amax/6 lands on an E4M3 tie only via fl(1/6)
        ],
        dtype=torch.float32,
    )
    return base


def main():
    cases = {}

    def add(name, x, gs=1.0, store_dtype="float32", keep_dequant=True):
        q, sf, sfl = quantize_nvfp4(x, gs)
        cases[f"{name}/x"] = x.float().numpy()
        cases[f"{name}/gs"] = np.array([gs], dtype=np.float64)
        cases[f"{name}/dtype"] = np.array(store_dtype)
        cases[f"{name}/packed"] = q.numpy()
        cases[f"{name}/sf_swizzled"] = sf.numpy()
        cases[f"{name}/sf_linear"] = sfl.numpy()
        if keep_dequant:
            cases[f"{name}/dequant"] = dequantize_nvfp4(q, sfl, gs).numpy()

    add("ties", ties_block())

    g = torch.Generator().manual_seed(0)
    x = torch.randn(256, 512, generator=g).to(torch.bfloat16)
    add("randn_bf16", x, store_dtype="bfloat16", keep_dequant=False)

    x = torch.randn(200, 320, generator=g)  # rows not a multiple of 128, K/16 = 20 not of 4
    amax = x.abs().max()
    gs = float(torch.tensor(2688.0) / amax)  # FP32 division, as the device path computes it
    add("randn_gs_f32", x, gs)

    x = torch.randn(128, 1024, generator=g)
    idx = torch.randperm(x.numel(), generator=g)[: x.numel() // 1000]
    sign = torch.where(torch.rand(idx.numel(), generator=g) < 0.5, -1.0, 1.0)
    x.view(-1)[idx] = 50.0 * sign
    x = x.to(torch.bfloat16)
    gs = float(torch.tensor(2688.0) / x.float().abs().max())
    add("outliers_bf16", x, gs, store_dtype="bfloat16", keep_dequant=False)

    x = (torch.randn(130, 96, generator=g) * 1e-3).to(torch.float16)
    add("small_f16", x, store_dtype="float16")

    x = torch.randn(64, 128, generator=g) * 2000.0  # scales overflow E4M3 -> NaN blocks
    add("overflow", x)

    # swizzle of an arbitrary scale grid (rows, cols not multiples of 128, 4)
    sf = torch.randint(0, 256, (300, 7), generator=g, dtype=torch.uint8)
    cases["swizzle/in"] = sf.numpy()
    cases["swizzle/out"] = swizzle_sf(sf).numpy()

    # small GEMM through the reference's own FP32 dequantised matmul (testing.py:18-27)
    m, n, k = 160, 192, 256
    a = torch.randn(m, k, generator=g)
    b = torch.randn(n, k, generator=g)
    aq, asf, asfl = quantize_nvfp4(a)
    bq, bsf, bsfl = quantize_nvfp4(b)
    c = dequantize_nvfp4(aq, asfl) @ dequantize_nvfp4(bq, bsfl).T
    cases.update({
        "gemm/a_packed": aq.numpy(), "gemm/b_packed": bq.numpy(),
        "gemm/a_sf": asf.numpy(), "gemm/b_sf": bsf.numpy(), "gemm/a_sf_linear": asfl.numpy(),
        "gemm/b_sf_linear": bsfl.numpy(), "gemm/c_fp32": c.numpy(),
    })

    np.savez_compressed(OUT, **cases)
    print(f"wrote {OUT}: {len(cases)} arrays, torch {torch.__version__}")


if __name__ == "__main__":
    sys.exit(main())
