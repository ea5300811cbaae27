"""Generate tests/golden/awq_golden.npz by running the REFERENCE implementation.

Run in a container that has the reference checked out (read-only is fine):

    python tests/golden/make_golden.py /path/to/reference

It imports the reference's own ``ashqk`` package (MMMchou/ash-quant-kernels) and
records, for small seeded cases:

- the format known-answer tests of tests/test_ref.py:17-38 (pack order, sign
  bit, round trip);
- ``quantize_awq`` / ``dequantize_awq`` outputs (ashqk/ref.py:58-86) for
  G in {32, 64, 128};
- GEMM cases on the shapes of tests/test_gemm.py:34-39 (plus a few more): the
  fp32 truth ``w4a16_gemm_fp32`` (ashqk/ref.py:95-103), the unfused fp16 path
  ``w4a16_gemm_ref`` (ashqk/ref.py:89-92), and the reference's Triton GEMV and
  v3 GEMM kernels run in the Triton CPU interpreter (TRITON_INTERPRET=1, the
  reference's own CI mode, .github/workflows/tests.yml:26-29).

The fixture travels with the repository; the reference does not.
"""

from __future__ import annotations

import os
import sys

os.environ["TRITON_INTERPRET"] = "1"  # must precede the first triton import

import numpy as np  # noqa: E402


def main(ref_root: str, out_path: str) -> None:
    sys.path.insert(0, ref_root)
    import torch
    import ashqk.ref as R
    from ashqk.kernels.w4a16_gemm_v3 import w4a16_gemm_v3
    from ashqk.kernels.w4a16_gemv import w4a16_gemv

    assert os.path.realpath(R.__file__).startswith(os.path.realpath(ref_root)), R.__file__
    out: dict[str, np.ndarray] = {}

    # --- format KATs (tests/test_ref.py:17-38) ---
    kat = torch.arange(1, 9, dtype=torch.int32).view(1, 8)
    out["kat_order_in"] = kat.numpy()
    out["kat_order_out"] = R.pack_awq(kat).numpy()
    sign = torch.full((2, 8), 15, dtype=torch.int32)
    out["kat_sign_in"] = sign.numpy()
    out["kat_sign_out"] = R.pack_awq(sign).numpy()
    g = torch.Generator().manual_seed(0)
    rt = torch.randint(0, 16, (64, 128), dtype=torch.int32, generator=g)
    out["roundtrip_in"] = rt.numpy()
    out["roundtrip_packed"] = R.pack_awq(rt).numpy()
    out["roundtrip_unpacked"] = R.unpack_awq(R.pack_awq(rt)).numpy()

    # --- quantise / dequantise (ashqk/ref.py:58-86) ---
    g = torch.Generator().manual_seed(1)
    w = torch.randn(256, 64, generator=g)
    out["quant_w"] = w.numpy()
    for gs in (32, 64, 128):
        qw, qz, s = R.quantize_awq(w, gs)
        out[f"quant_g{gs}_qweight"] = qw.numpy()
        out[f"quant_g{gs}_qzeros"] = qz.numpy()
        out[f"quant_g{gs}_scales"] = s.numpy()
        out[f"quant_g{gs}_deq_f32"] = R.dequantize_awq(qw, qz, s).numpy()
        out[f"quant_g{gs}_deq_f16"] = R.dequantize_awq(qw, qz, s, torch.float16).numpy()

    # --- GEMM cases ---
    shapes = [(1, 64, 256), (7, 72, 256), (17, 128, 384), (2, 64, 256), (16, 256, 1024), (4, 136, 512)]
    names = []
    for ci, (m, n, k) in enumerate(shapes):
        for gs in (32, 64, 128):
            if k % gs:
                continue
            g = torch.Generator().manual_seed(100 + ci * 10 + gs)
            x = torch.randn(m, k, generator=g).to(torch.float16)
            wt = torch.randn(k, n, generator=g) * 0.02
            qw, qz, s = R.quantize_awq(wt, gs)
            name = f"gemm_m{m}_n{n}_k{k}_g{gs}"
            names.append(name)
            out[name + "_x"] = x.numpy()
            out[name + "_qweight"] = qw.numpy()
            out[name + "_qzeros"] = qz.numpy()
            out[name + "_scales"] = s.numpy()
            out[name + "_y_fp32"] = R.w4a16_gemm_fp32(x, qw, qz, s).numpy()
            out[name + "_y_ref"] = R.w4a16_gemm_ref(x, qw, qz, s).numpy()
            out[name + "_y_gemv"] = w4a16_gemv(x, qw, qz, s).numpy()
            out[name + "_y_v3"] = w4a16_gemm_v3(x, qw, qz, s).numpy()
            print(name, flush=True)
    out["gemm_cases"] = np.array(names)
    np.savez_compressed(out_path, **out)
    print("wrote", out_path, os.path.getsize(out_path), "bytes")


if __name__ == "__main__":
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("ASHQK_REFERENCE", "")
    if not ref or not os.path.isdir(os.path.join(ref, "ashqk")):
        sys.exit("usage: make_golden.py <reference checkout containing ashqk/>")
    main(ref, os.path.join(os.path.dirname(os.path.abspath(__file__)), "awq_golden.npz"))
