"""Load the committed golden fixtures (tests/golden/*.npz) as torch tensors."""

from pathlib import Path

import numpy as np
import torch

GOLDEN = Path(__file__).resolve().parent / "golden"


def bits(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.uint16).view(np.int16)).view(torch.bfloat16)


def load(name: str) -> dict:
    with np.load(GOLDEN / f"{name}.npz") as z:
        return {k: z[k] for k in z.files}


def attention_case(name: str):
    """(q [B,32,128], k [B,8,cap,128], v, lens) with K/V unpacked into a zero-padded cache."""
    z = load("attention")
    lens = [int(x) for x in z[f"{name}_lens"]]
    q = bits(z[f"{name}_q"])
    kp, vp = bits(z[f"{name}_k"]), bits(z[f"{name}_v"])
    B, cap = len(lens), max(lens)
    k = torch.zeros(B, kp.shape[0], cap, kp.shape[2], dtype=torch.bfloat16)
    v = torch.zeros_like(k)
    o = 0
    for b, L in enumerate(lens):
        k[b, :, :L] = kp[:, o:o + L]
        v[b, :, :L] = vp[:, o:o + L]
        o += L
    return q, k, v, lens, torch.from_numpy(z[f"{name}_out_gqa"]), torch.from_numpy(z[f"{name}_out_rep"])
