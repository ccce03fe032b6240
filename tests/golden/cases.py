"""Seeded recipes for the golden cases (shared by the generator and the tests)."""
from __future__ import annotations

import torch

SKEW_LOCAL_EXPERTS = (0, 8, 16, 24)


def adversarial_logits():
    """Hand-built routing stress rows: exact ties, saturated sigmoids, bias spikes."""
    g = torch.Generator().manual_seed(7)
    rows = []
    rows.append(torch.zeros(256))                            # every score equal
    rows.append(torch.full((256,), 30.0))                    # sigmoid saturates to 1.0
    r = torch.randn(256, generator=g); r[::2] = 0.5; rows.append(r)   # many equal values
    r = torch.randn(256, generator=g) * 20; rows.append(r)  # mostly saturated 0 / 1
    r = torch.randn(256, generator=g); r[32:64] = 40.0; rows.append(r)  # one group saturated
    r = torch.randn(256, generator=g); r[0:8] = 2.0; r[40:48] = 2.0; rows.append(r)  # tied top-8 across groups
    for _ in range(26):
        r = torch.randn(256, generator=g)
        k = int(torch.randint(0, 256, (1,), generator=g))
        r[k:k + 3] = r[k]                                     # local duplicates
        rows.append(r)
    return torch.stack(rows).float()


def routing_case(name):
    """Return (logits f32 [T, 256], bias bf16 [256]) for a named routing case."""
    if name == "routing_T16384_seed11":
        g = torch.Generator().manual_seed(11)
        logits = torch.randn(16384, 256, generator=g)
        bias = (torch.randn(256, generator=g) * 0.1).to(torch.bfloat16)
    elif name == "routing_T4096_seed12_skewed":
        g = torch.Generator().manual_seed(12)
        logits = torch.randn(4096, 256, generator=g)
        b = torch.randn(256, generator=g) * 0.1
        for le in SKEW_LOCAL_EXPERTS:
            b[le] = 3.0
        bias = b.to(torch.bfloat16)
    elif name == "routing_adversarial":
        logits = adversarial_logits()
        g = torch.Generator().manual_seed(13)
        b = torch.randn(256, generator=g) * 0.1
        b[100] = 3.0
        bias = b.to(torch.bfloat16)
    else:
        raise KeyError(name)
    return logits.float(), bias


ROUTING_CASES = ("routing_T16384_seed11", "routing_T4096_seed12_skewed", "routing_adversarial")
FULL_CASES = {  # name: (T, seed, skewed)
    "full_T16_seed0": (16, 0, False),
    "full_T1_seed3": (1, 3, False),
    "full_T3_seed5": (3, 5, False),
    "full_T1_seed16": (1, 16, False),
    "full_T16_seed1_skewed": (16, 1, True),
}
