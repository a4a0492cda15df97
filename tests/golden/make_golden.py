"""Generate the golden fixtures by running the REFERENCE's own Python code.

Run in a container where the reference checkout is readable (it is not needed
at test time; the fixtures are committed):

    python tests/golden/make_golden.py /path/to/ComfyUI-AppleSilicon-Optimized

What is pinned, and how:
  fp8_lut.npz       _patches/_common.py fp8_to_float_lut (all 256 codes, e4m3fn + e5m2)
  int8_epilogue.npz _patches/int8_linear_kernel_mps.py _int8_linear_prequant, chunked
                    epilogue branch (:203-215), driven with a stand-in native module whose
                    only method is an exact int64 i8_matmul2d_nt (so the reference's own
                    rescale / cast / bias code produces the bytes)
  fp8_fast.npz      _patches/scaled_mm_fp8.py _fast_route (:123-146), driven with a
                    stand-in backend whose fp8fp8_matmul2d_nt is an exact fp64 product, so
                    the reference's own scale/bias/cast order produces the values
Inputs are seeded; the stand-ins compute exact integer / fp64 products only.
"""
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _exact_int_mm(a, b_nk):
    return (a.long() @ b_nk.long().t()).to(torch.int32)


class _ChunkedOnlyInt8:
    """Exposes only i8_matmul2d_nt -> the reference takes its chunked epilogue."""

    @staticmethod
    def i8_matmul2d_nt(a, b):
        return _exact_int_mm(a, b)


class _ExactFp8Backend:
    @staticmethod
    def fp8fp8_matmul2d_nt(a_u8, w_u8, K, N):
        a = a_u8.view(torch.float8_e4m3fn).to(torch.float64)
        w = w_u8.view(torch.float8_e4m3fn).to(torch.float64)
        return (a @ w.t()).to(torch.float32)


def main(ref_root):
    sys.path.insert(0, ref_root)
    from _patches import _common, int8_linear_kernel_mps as k8, scaled_mm_fp8 as s8

    # 1) FP8 decode table
    lut = {}
    for name, dt in (("e4m3fn", torch.float8_e4m3fn), ("e5m2", torch.float8_e5m2)):
        t = _common.fp8_to_float_lut(dt, torch.device("cpu"), torch.float32)
        lut[name] = t.numpy().view(np.uint32)
    np.savez_compressed(os.path.join(HERE, "fp8_lut.npz"), **lut)

    # 2) INT8 chunked dequant epilogue (reference code, exact int GEMM)
    g = torch.Generator().manual_seed(11)
    cases = {}
    k8._kernel = _ChunkedOnlyInt8()
    for i, (M, K, N, ws_kind, bias) in enumerate(((64, 256, 96, "channel", True),
                                                  (33, 512, 129, "scalar", True),
                                                  (17, 128, 64, "channel", False))):
        x8 = torch.randint(-128, 128, (M, K), generator=g, dtype=torch.int8)
        xs = torch.rand(M, 1, generator=g) * 0.02 + 1e-4
        w = torch.randint(-128, 128, (N, K), generator=g, dtype=torch.int8)
        ws = torch.rand(N if ws_kind == "channel" else 1, 1, generator=g) * 0.01 + 0.001
        b = torch.randn(N, generator=g).to(torch.bfloat16) if bias else None
        # out_dtype float32 would skip bf16; the reference's chunked branch is the one
        # taken for any out_dtype when the fused entry points are absent.
        out = k8._int8_linear_prequant(x8, xs, w, ws, b, torch.bfloat16, (M, K))
        cases[f"c{i}_x8"] = x8.numpy()
        cases[f"c{i}_xs"] = xs.numpy()
        cases[f"c{i}_w"] = w.numpy()
        cases[f"c{i}_ws"] = ws.numpy()
        cases[f"c{i}_bias"] = (b.float().numpy() if b is not None else np.zeros(0, np.float32))
        cases[f"c{i}_out_bits"] = out.contiguous().view(torch.int16).numpy()
    np.savez_compressed(os.path.join(HERE, "int8_epilogue.npz"), **cases)

    # 3) FP8 fast-route epilogue (reference code, exact product)
    s8._backend = _ExactFp8Backend()
    g = torch.Generator().manual_seed(2)
    f = {}
    for i, (M, K, N, per_row) in enumerate(((48, 256, 80, False), (20, 128, 40, True))):
        a = (torch.randn(M, K, generator=g) * 0.3).to(torch.float8_e4m3fn)
        w = (torch.randn(N, K, generator=g) * 0.3).to(torch.float8_e4m3fn)
        sa = torch.rand(M, 1, generator=g) * 0.1 + 0.01 if per_row else torch.tensor(0.02)
        sb = torch.tensor(0.05)
        b = (torch.randn(N, generator=g) * 0.01).to(torch.bfloat16)
        out = s8._fast_route(a, w.t(), sa, sb, None, b, torch.float32)
        f[f"c{i}_a"] = a.view(torch.uint8).numpy()
        f[f"c{i}_w"] = w.view(torch.uint8).numpy()
        f[f"c{i}_sa"] = sa.reshape(-1).numpy()
        f[f"c{i}_sb"] = sb.reshape(-1).numpy()
        f[f"c{i}_bias"] = b.float().numpy()
        f[f"c{i}_out"] = out.numpy()
    np.savez_compressed(os.path.join(HERE, "fp8_fast.npz"), **f)
    print("wrote", sorted(os.listdir(HERE)))


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("REFERENCE_ROOT", ""))
