"""Generates tests/golden/attention_*.npz from the reference's sdpa_reference.

Runs ONLY where the reference checkout is present (pass its root with
--reference; default: the REFERENCE_ROOT environment variable). The GPU host
never runs this: the committed .npz files travel instead.

What is taken from the reference, unmodified: sdpa_reference from
kernels/attention/common.py (lines 115-138), extracted with `ast` and executed
on the CPU in fp32 (the module itself imports Triton's Gluon front end, which
the reference only uses on an AMD GPU). Inputs are seeded standard normals
rounded to the problem's 16-bit type, in the bhsd frame the function expects;
each file holds q, k, v (16-bit bit patterns), the reference output o_ref
(fp32) and the problem's sizes.

    python tests/golden/make_attention_golden.py --reference <path to checkout>
"""

from __future__ import annotations

import argparse
import ast
import math
import os

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
COMMON = os.path.join("kernels", "attention", "common.py")

# (name, B, HQ, HK, Sq, Sk, D, dtype)
CASES = [
    ("attention_f16_b1h4k2_s128_d64", 1, 4, 2, 128, 128, 64, torch.float16),
    ("attention_bf16_b2h2k2_q100_k200_d128", 2, 2, 2, 100, 200, 128, torch.bfloat16),
    ("attention_bf16_b1h4k1_s256_d128", 1, 4, 1, 256, 256, 128, torch.bfloat16),
    ("attention_f16_b1h2k1_q192_k320_d128", 1, 2, 1, 192, 320, 128, torch.float16),
]


def load_sdpa_reference(ref_root: str):
    src_path = os.path.join(ref_root, COMMON)
    tree = ast.parse(open(src_path).read(), filename=src_path)
    body = [n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name == "sdpa_reference"]
    if not body:
        raise RuntimeError("sdpa_reference not found")
    ns = {"torch": torch, "math": math}
    exec(compile(ast.Module(body=body, type_ignores=[]), src_path, "exec"), ns)
    return ns["sdpa_reference"]


def bits16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--reference", default=os.environ.get("REFERENCE_ROOT"))
    args = ap.parse_args()
    if not args.reference:
        raise SystemExit("pass --reference <reference checkout>")
    sdpa_reference = load_sdpa_reference(args.reference)
    for i, (name, B, HQ, HK, Sq, Sk, D, dt) in enumerate(CASES):
        g = torch.Generator().manual_seed(1000 + i)
        q = torch.randn((B, HQ, Sq, D), generator=g).to(dt)
        k = torch.randn((B, HK, Sk, D), generator=g).to(dt)
        v = torch.randn((B, HK, Sk, D), generator=g).to(dt)
        sm_scale = D ** -0.5
        o_ref = sdpa_reference(q, k, v, causal=False, sm_scale=sm_scale)
        np.savez_compressed(
            os.path.join(HERE, name + ".npz"),
            q=bits16(q), k=bits16(k), v=bits16(v), o_ref=o_ref.numpy().astype(np.float32),
            dims=np.array([B, HQ, HK, Sq, Sk, D], dtype=np.int64),
            dtype=np.array(str(dt).split(".")[-1]), sm_scale=np.array(sm_scale),
        )
        print(name, tuple(o_ref.shape))


if __name__ == "__main__":
    main()
