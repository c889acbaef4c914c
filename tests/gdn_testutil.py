"""Shared helpers for the parity tests: seeded inputs with the shapes and
distributions of the benchmark configurations, and the tolerance metrics."""

from __future__ import annotations

import numpy as np
import torch

# Tolerances against an fp64 evaluation of the same (rounded) inputs.
FP32_REL_RMS = 1e-4
BF16_REL_RMS = 1e-2
BF16_MAX_ABS = 2e-2


def rel_rms(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.sqrt(np.mean((a - b) ** 2)) / (np.sqrt(np.mean(b ** 2)) + 1e-30))


def max_abs(a, b) -> float:
    return float(np.max(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64))))


def make_inputs(seed, B, T, H, HV, K, V, dtype=torch.bfloat16, device="cuda", nseq_state=None,
                state_std=0.0):
    """q, k, v ~ N(0,1) in `dtype`; g = logsigmoid(N(0,1)), beta = sigmoid(N(0,1))
    in fp32; optional initial states ~ N(0, state_std)."""
    gen = torch.Generator().manual_seed(seed)
    q = torch.randn(B, T, H, K, generator=gen).to(dtype)
    k = torch.randn(B, T, H, K, generator=gen).to(dtype)
    v = torch.randn(B, T, HV, V, generator=gen).to(dtype)
    g = torch.nn.functional.logsigmoid(torch.randn(B, T, HV, generator=gen))
    beta = torch.sigmoid(torch.randn(B, T, HV, generator=gen))
    h0 = None
    if nseq_state:
        h0 = torch.randn(nseq_state, HV, K, V, generator=gen) * state_std
    out = [q, k, v, g, beta, h0]
    return [None if x is None else x.to(device) for x in out]


def np64(t):
    return None if t is None else t.detach().float().cpu().numpy().astype(np.float64)
