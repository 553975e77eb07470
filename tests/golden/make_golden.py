"""Generates the golden vectors in tests/golden/golden.npz by running the reference's own code.

Run where the byteprof project is checked out, naming its root with --ref or $BYTEPROF_REF:

    TRITON_INTERPRET=1 python tests/golden/make_golden.py --ref <path to byteprof checkout>

What it runs (paths inside the byteprof project):
  * byteprof/quant/triton_int8.py:50-55  quantize_rowwise_int8 on seeded bf16 weights (torch, CPU)
  * byteprof/optim/skinny.py:209-217     dequantize, and the fp32 dequantize-then-matmul reference of
                                         tests/test_skinny.py:38 (torch, CPU)
  * byteprof/optim/skinny.py:172-206     quantize_int4, pack_int4 (R = 32 and 16), unpack_int4 and the
                                         int4 dequantizer (torch, CPU). The Triton int4 kernel itself is not
                                         run: under the CPU interpreter its bit-cast of the nibbles into fp32
                                         gives wrong values, so kernel parity rests on the fp32 reference.
  * byteprof/quant/triton_int8.py:15-47  the Triton int8 GEMV, under the Triton CPU interpreter
  * byteprof/optim/mlstm_multistep.py    multistep_fw_kernel and lazy_commit_kernel with fp32 inputs
                                         (the interpreter has no bf16), and accept_kernel, under
                                         the interpreter, launched directly with BQ = DQ or DQ / 2
                                         (the wrapper's block heuristic lives in the missing
                                         mlstm_kernels package)
The arrays hold bf16 tensors as their uint16 bit patterns. Nothing at test time reads the reference.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

os.environ.setdefault("TRITON_INTERPRET", "1")

import numpy as np  # noqa: E402
import torch  # noqa: E402

OUT = Path(__file__).resolve().parent / "golden.npz"


def reference_root(argv: list[str]) -> Path:
    """The byteprof checkout: --ref PATH, else $BYTEPROF_REF; there is no default."""
    import argparse

    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("BYTEPROF_REF"))
    a = ap.parse_args(argv)
    if not a.ref:
        ap.error("name the byteprof checkout with --ref or $BYTEPROF_REF")
    root = Path(a.ref)
    if not (root / "byteprof").is_dir():
        ap.error(f"{root} holds no byteprof package")
    return root


def bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def main(argv: list[str] | None = None) -> None:
    sys.path.insert(0, str(reference_root(sys.argv[1:] if argv is None else argv)))
    import triton
    import triton.language as tl

    from byteprof.optim import mlstm_multistep as ms
    from byteprof.optim import skinny as S
    from byteprof.quant import triton_int8 as Q

    g: dict[str, np.ndarray] = {}

    # ---- int8 quantizer and dequantizer ------------------------------------------------------------
    gen = torch.Generator().manual_seed(1234)
    w = (torch.randn(48, 384, generator=gen) * 0.02).to(torch.bfloat16)
    w[3] = 0  # an all-zero row exercises the 1e-12 clamp
    w[7, :5] = torch.tensor([1e-3, -2e-3, 0.5, -0.5, 0.25], dtype=torch.bfloat16)
    q, s = Q.quantize_rowwise_int8(w)
    g["q8_w"], g["q8_q"], g["q8_scale"] = bits(w), q.numpy().copy(), bits(s)
    g["q8_deq"] = S.dequantize("int8", q, s).numpy().copy()

    # ---- int4 group quantizer, packing, dequantizer -------------------------------------------------
    gen = torch.Generator().manual_seed(4444)
    w4 = (torch.randn(40, 384, generator=gen) * 0.03).to(torch.bfloat16)
    w4[5] = 0  # an all-zero row: scale clamped at 1e-6, zero -0
    w4[9, 130:136] = torch.tensor([0.9, -0.8, 0.7, 1e-4, -1e-4, 0.0], dtype=torch.bfloat16)  # a wide group
    g["q4_w"] = bits(w4)
    for r in (32, 16):
        packed, scale4, zero4 = S.quantize_int4(w4, tile_rows=r)
        g[f"q4_r{r}_packed"], g[f"q4_r{r}_scale"], g[f"q4_r{r}_zero"] = packed.numpy().copy(), bits(scale4), bits(zero4)
        g[f"q4_r{r}_codes"] = S.unpack_int4(packed, 40).numpy().copy()
        g[f"q4_r{r}_deq"] = S.dequantize("int4", packed, scale4, zero4).numpy().copy()
    x4 = torch.randn(5, 384, generator=gen).to(torch.bfloat16)
    g["q4lin_x"] = bits(x4)
    g["q4lin_y"] = (x4.float() @ S.dequantize("int4", *S.quantize_int4(w4)).T).numpy().copy()

    # ---- fp32 dequantize-then-matmul reference (the reference tests' oracle) -------------------------
    for kind, (n, k), m in (("bf16", (70, 384), 3), ("int8", (37, 256), 5), ("bf16", (129, 640), 17)):
        gen = torch.Generator().manual_seed(n * 1000 + k)
        wb = (torch.randn(n, k, generator=gen) * 0.02).to(torch.bfloat16)
        x = torch.randn(m, k, generator=gen).to(torch.bfloat16)
        args = (wb,) if kind == "bf16" else Q.quantize_rowwise_int8(wb)
        ref_w = S.dequantize(kind, *args)
        y = x.float() @ ref_w.T
        key = f"lin_{kind}_{n}x{k}_m{m}"
        g[key + "_x"], g[key + "_w"], g[key + "_y"] = bits(x), bits(wb), y.numpy().copy()

    # ---- Triton int8 GEMV under the interpreter -------------------------------------------------------
    for n, k in ((24, 128), (37, 1000), (3, 129)):
        gen = torch.Generator().manual_seed(7 * n + k)
        wb = (torch.randn(n, k, generator=gen) * 0.05).to(torch.bfloat16)
        qq, ss = Q.quantize_rowwise_int8(wb)
        x = torch.randn(1, k, generator=gen).to(torch.bfloat16)
        y = Q.gemv_int8(x, qq, ss)
        key = f"gemv_{n}x{k}"
        g[key + "_x"], g[key + "_q"], g[key + "_scale"], g[key + "_y"] = bits(x), qq.numpy().copy(), bits(ss), bits(y)

    # ---- fused mLSTM kernels, fp32, under the interpreter ----------------------------------------------
    for nh, dq, bq, dv, t in ((2, 64, 64, 32, 5), (2, 128, 64, 32, 4), (1, 512, 256, 16, 3)):
        gen = torch.Generator().manual_seed(nh * 100 + dq + t)
        r = lambda *shape: torch.randn(*shape, generator=gen)  # noqa: E731
        qv, kv, vv = r(t, nh, dq), r(t, nh, dq), r(t, nh, dv)
        iv, fv = r(t, nh, 1) * 2, r(t, nh, 1) * 2
        c0, n0, m0 = r(1, nh, dq, dv) * 0.1, r(1, nh, dq) * 0.1, r(1, nh, 1)
        h = torch.zeros(t, nh, dv)
        ns, msv = torch.zeros(nh, dq), torch.zeros(nh)
        bv = 16
        ms.multistep_fw_kernel[(dv // bv, nh)](
            c0, n0, m0, qv, kv, vv, iv, fv, h, ns, msv, t, qv.stride(0), vv.stride(0), iv.stride(0), h.stride(0),
            qk_scale=dq ** -0.5, NH=nh, DQ=dq, DV=dv, BQ=bq, BV=bv, EPS=1e-6, DTYPE=tl.float32,
            DTYPE_STATE=tl.float32, num_warps=1)
        key = f"ms_nh{nh}_dq{dq}_dv{dv}_t{t}"
        for name, arr in (("q", qv), ("k", kv), ("v", vv), ("i", iv), ("f", fv), ("c0", c0), ("n0", n0), ("m0", m0),
                          ("h", h), ("nstart", ns), ("mstart", msv)):
            g[f"{key}_{name}"] = arr.numpy().copy()
        for length in range(t):
            cur = (c0.clone(), n0.clone(), m0.clone())
            ms.lazy_commit_kernel[(dv // bv, nh)](
                cur[0], cur[1], cur[2], ns, msv, kv, vv, iv, fv, torch.tensor(length), kv.stride(0), vv.stride(0),
                iv.stride(0), NH=nh, DQ=dq, DV=dv, BQ=bq, BV=bv, DTYPE=tl.float32, DTYPE_STATE=tl.float32,
                num_warps=2)
            for name, arr in zip(("c", "n", "m"), cur):
                g[f"{key}_L{length}_{name}"] = arr.numpy().copy()

    # ---- accept kernel known answers ---------------------------------------------------------------
    ids = torch.tensor([10, 5, 6, 7, 8, 9])
    toks = ([5, 6, 99, 8, 9, 3], [5, 6, 7, 8, 9 + 260, 3], [1, 6, 7, 8, 9, 3], [5, 6, 7, 8, 9, 3])
    g["acc_ids"] = ids.numpy().copy()
    for j, tokl in enumerate(toks):
        tok = torch.tensor(tokl)
        out = torch.zeros(8, dtype=torch.long)
        ms.accept_kernel[(1,)](ids, tok, out, S=6, SMAX=6, num_warps=1)
        g[f"acc_tok{j}"], g[f"acc_out{j}"] = tok.numpy().copy(), out.numpy().copy()

    g["meta_triton"] = np.array(triton.__version__)
    g["meta_torch"] = np.array(torch.__version__)
    np.savez_compressed(OUT, **g)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes, {len(g)} arrays)")


if __name__ == "__main__":
    main()
