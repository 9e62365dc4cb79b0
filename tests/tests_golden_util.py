"""Decoding of tests/golden/ref_kernel_cases.npz (helper for the tests)."""
import numpy as np
import torch


def decode_case(z, name):
    b, s, h, d, causal, seed = (int(x) for x in z[f"{name}__meta"])
    dt = str(z[f"{name}__dtype"])
    bits = torch.from_numpy(np.ascontiguousarray(z[f"{name}__o_bits"]))
    o = bits.view(getattr(torch, dt)).to(torch.float32).numpy()
    return b, s, h, d, bool(causal), seed, dt, o
