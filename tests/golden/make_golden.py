"""Generates the golden vectors under tests/golden/ from the reference itself.

Runs ONLY where the reference checkout is present (pass its root with
--reference; default: the REFERENCE_ROOT environment variable). The GPU host
never runs this: the committed .npz files travel instead.

What is taken from the reference, unmodified:
  - mxfp4_to_f32, e8m0_to_f32, generate_mxfp4_inputs, torch_reference and
    SCALE_GROUP_SIZE from kernels/gemm/intra_wave/a4w4/bench.py (lines 77-164),
    extracted with `ast` and executed with DEVICE = "cpu" (the module itself
    cannot be imported without an AMD GPU: it resolves a Triton device at
    import time, bench.py:74).
The a16w16 and a8w8 reference checks are one-line torch expressions inside
test_correctness (kernels/gemm/intra_wave/a16w16/bench.py:174-183,
kernels/gemm/intra_wave/a8w8/bench.py:133-138); they are evaluated here on the
CPU with the same input recipe. The e5m2 table is torch's own
float -> float8_e5m2 cast of a set of fp32 probe values.

    python tests/golden/make_golden.py --reference <path to checkout>
"""

from __future__ import annotations

import argparse
import ast
import os

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
A4W4_BENCH = os.path.join("kernels", "gemm", "intra_wave", "a4w4", "bench.py")
WANTED = {"mxfp4_to_f32", "e8m0_to_f32", "generate_mxfp4_inputs", "torch_reference"}


def load_reference_helpers(ref_root: str) -> dict:
    src_path = os.path.join(ref_root, A4W4_BENCH)
    tree = ast.parse(open(src_path).read(), filename=src_path)
    body = []
    for node in tree.body:
        if isinstance(node, ast.FunctionDef) and node.name in WANTED:
            body.append(node)
        elif isinstance(node, ast.Assign) and any(
                isinstance(t, ast.Name) and t.id == "SCALE_GROUP_SIZE" for t in node.targets):
            body.append(node)
    mod = ast.Module(body=body, type_ignores=[])
    ns = {"torch": torch, "DEVICE": "cpu"}
    exec(compile(mod, src_path, "exec"), ns)
    missing = WANTED - set(ns)
    if missing:
        raise RuntimeError(f"reference helpers not found: {missing}")
    return ns


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def e5m2_probe_values() -> np.ndarray:
    rng = np.random.default_rng(7)
    vals = [
        rng.standard_normal(4096).astype(np.float32),
        (rng.standard_normal(2048) * 1e4).astype(np.float32),
        (rng.standard_normal(2048) * 1e-5).astype(np.float32),
        np.ldexp(rng.uniform(1, 2, 1024), rng.integers(-30, 18, 1024)).astype(np.float32),
    ]
    edges = []
    # every e5m2 value, the midpoints between neighbours and values just around them
    allq = torch.arange(256, dtype=torch.int32).to(torch.uint8).view(torch.float8_e5m2)
    fin = allq.float().numpy()
    fin = np.unique(fin[np.isfinite(fin)])
    mids = (fin[:-1].astype(np.float64) + fin[1:]) / 2
    for m in mids.astype(np.float32):
        edges += [m, np.nextafter(m, np.float32(np.inf)), np.nextafter(m, np.float32(-np.inf))]
    edges += list(fin)
    edges += [0.0, -0.0, 57344.0, 61440.0, 61439.996, 65504.0, 1e30, -1e30,
              np.inf, -np.inf, np.nan, 2.0 ** -16, 2.0 ** -17, 2.0 ** -18, 1.5 * 2.0 ** -17,
              2.0 ** -14, np.float32(1e-45), np.float32(-1e-45)]
    vals.append(np.array(edges, dtype=np.float32))
    return np.concatenate(vals).astype(np.float32)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--reference", default=os.environ.get("REFERENCE_ROOT"))
    args = ap.parse_args()
    if not args.reference or not os.path.isdir(args.reference):
        raise SystemExit("pass --reference <path of the reference checkout>")
    ns = load_reference_helpers(args.reference)

    # --- decode tables: every byte through the reference's decoders
    allb = torch.arange(256, dtype=torch.int32).to(torch.uint8).reshape(1, 256)
    dec_fp4 = ns["mxfp4_to_f32"](allb.clone()).numpy()          # (1, 512)
    dec_e8m0 = ns["e8m0_to_f32"](allb.clone().reshape(256)).numpy()
    np.savez_compressed(os.path.join(HERE, "decode_tables.npz"), bytes=allb.numpy()[0],
                        mxfp4=dec_fp4[0], e8m0=dec_e8m0)

    # --- MXFP4 GEMM: the reference's generator (seed 42) and torch_reference
    for (M, N, K) in [(128, 256, 256), (256, 256, 512), (200, 320, 1024)]:
        a, b, sa, sb = ns["generate_mxfp4_inputs"](M, N, K)
        c = ns["torch_reference"](a, b, sa, sb, dtype=torch.bfloat16)
        np.savez_compressed(
            os.path.join(HERE, f"mxfp4_ref_{M}x{N}x{K}.npz"), a=a.numpy(), b=b.numpy(),
            a_scales=sa.contiguous().numpy(), b_scales=sb.contiguous().numpy(),
            a_scales_strides=np.array(sa.stride()), c_bf16=bf16_bits(c))

    # --- a16w16: torch.matmul(a, b) in the input dtype, rand - 0.5 inputs
    for dt, name in [(torch.float16, "f16"), (torch.bfloat16, "bf16")]:
        g = torch.Generator().manual_seed(3)
        M, N, K = 128, 256, 320
        a = torch.rand((M, K), generator=g, dtype=torch.float32).to(dt) - 0.5
        b = torch.rand((N, K), generator=g, dtype=torch.float32).to(dt).T - 0.5
        c = torch.matmul(a, b)
        bt = b.T.contiguous()
        if dt == torch.float16:
            arrs = dict(a=a.numpy(), b_t=bt.numpy(), c=c.numpy())
        else:
            arrs = dict(a=bf16_bits(a), b_t=bf16_bits(bt), c=bf16_bits(c))
        np.savez_compressed(os.path.join(HERE, f"a16w16_{name}_{M}x{N}x{K}.npz"), **arrs)

    # --- a8w8: (rand - 0.5).to(e5m2), torch.matmul(a.to(f16), b.to(f16))
    g = torch.Generator().manual_seed(5)
    M, N, K = 128, 256, 512
    a = (torch.rand((M, K), generator=g, dtype=torch.float32).half() - 0.5).to(torch.float8_e5m2)
    b = (torch.rand((N, K), generator=g, dtype=torch.float32).half().T - 0.5).to(
        torch.float8_e5m2)
    c = torch.matmul(a.to(torch.float16), b.to(torch.float16))
    np.savez_compressed(os.path.join(HERE, f"a8w8_e5m2_{M}x{N}x{K}.npz"),
                        a=a.view(torch.uint8).numpy(),
                        b_t=b.T.contiguous().view(torch.uint8).numpy(), c=c.numpy())

    # --- torch's fp32 -> float8_e5m2 rounding
    x = e5m2_probe_values()
    q = torch.from_numpy(x).to(torch.float8_e5m2).view(torch.uint8).numpy()
    np.savez_compressed(os.path.join(HERE, "e5m2_cast.npz"), x=x, q=q)
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    main()
