"""Generate golden vectors from the REFERENCE kernel itself.

Runs on a B200 box: imports the reference extension built from the
reference's own sources by oracle/build_ref.py (oracle/_ref/), feeds it
seeded inputs (oracle.attention_oracle.make_inputs, CPU generator) and saves
its outputs with a digest of the inputs:

    python tests/golden/make_golden.py --out tests/golden/ref_kernel_cases.npz

Inputs are not stored; tests regenerate them from the seed and check the
digest.  The reference only supports seqlen % 64 == 0, head_dim 64/128,
heads_k == heads (csrc/flash_fwd_kernel.cuh:53,130-154; flash_api.cpp:28-29)
and returns O only, so these cases stay inside that envelope.
"""
from __future__ import annotations

import argparse
import hashlib
import os
import sys

import numpy as np
import torch

REPO = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, REPO)

from oracle.attention_oracle import make_inputs  # noqa: E402
from oracle.build_ref import load_module  # noqa: E402

# (name, batch, seqlen, heads, head_dim, dtype, causal, seed)
CASES = [
    ("fp16_d64_nc", 1, 128, 2, 64, "float16", False, 101),
    ("fp16_d64_c", 1, 128, 2, 64, "float16", True, 102),
    ("bf16_d128_nc", 1, 128, 2, 128, "bfloat16", False, 103),
    ("bf16_d128_c", 1, 128, 2, 128, "bfloat16", True, 104),
    ("bf16_d64_c_s192", 1, 192, 1, 64, "bfloat16", True, 105),
    ("fp16_d128_nc_s192", 1, 192, 1, 128, "float16", False, 106),
    ("fp16_d64_c_b2_s256", 2, 256, 1, 64, "float16", True, 107),
    ("bf16_d64_nc_b2_s256", 2, 256, 1, 64, "bfloat16", False, 108),
]


def digest(*tensors: torch.Tensor) -> str:
    h = hashlib.sha256()
    for t in tensors:
        h.update(t.contiguous().view(torch.int16).numpy().tobytes())
    return h.hexdigest()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=os.path.join(os.path.dirname(os.path.abspath(__file__)), "ref_kernel_cases.npz"))
    a = ap.parse_args()
    ref = load_module()
    out = {}
    for name, b, s, h, d, dt, causal, seed in CASES:
        dtype = getattr(torch, dt)
        q, k, v = make_inputs(b, s, h, d, dtype, seed=seed)
        o = ref.forward(q.cuda(), k.cuda(), v.cuda(), causal)
        torch.cuda.synchronize()
        out[f"{name}__o_bits"] = o.cpu().contiguous().view(torch.int16).numpy()
        out[f"{name}__meta"] = np.array([b, s, h, d, int(causal), seed], dtype=np.int64)
        out[f"{name}__dtype"] = np.array(dt)
        out[f"{name}__digest"] = np.array(digest(q, k, v))
        print(name, "done", flush=True)
    os.makedirs(os.path.dirname(a.out), exist_ok=True)
    np.savez_compressed(a.out, **out)
    print("wrote", a.out)


if __name__ == "__main__":
    main()
