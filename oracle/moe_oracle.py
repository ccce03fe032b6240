"""CPU oracle for the DeepSeek-V3 FP8 block-scale fused MoE (numpy restatement).

TEST INFRASTRUCTURE ONLY. Only `tests/`, `__graft_entry__.smoke()` and the
`cpu_baseline` / `--impl reference` legs of `bench.py` may import this module,
and only as the checker or the timed CPU baseline. The product path never
calls into it.

It restates, in numpy, the operator's reference implementation: the
`reference` source embedded in
`resources/moe_fp8_block_scale_ds_routing_topk8_ng8_kg4_e32_h7168_i2048.json:146`
(the definition file's only code). Each function below names the step of that
source it follows. The restatement is pinned against golden vectors produced by
running the reference itself (`tests/golden/make_golden.py`).

Differences that do not change results:
* by default only the experts that some token selects are dequantised (the
  reference dequantises all of them first; `dequant_all=True` does the same, for
  timing the reference's cost);
* fp32 matmuls go through numpy/BLAS rather than torch; the summation order of
  the fp32 dot products differs, which is far below the test tolerances.
"""
from __future__ import annotations

import numpy as np

H = 7168
I = 2048
E_GLOBAL = 256
TOP_K = 8
N_GROUP = 8
TOPK_GROUP = 4
BLOCK = 128


def _e4m3_table() -> np.ndarray:
    """Value of every float8 e4m3fn byte (1 sign, 4 exponent bits with bias 7,
    3 mantissa bits, no infinities, 0x7f/0xff are NaN)."""
    tab = np.zeros(256, dtype=np.float32)
    for b in range(256):
        sign = -1.0 if b & 0x80 else 1.0
        exp = (b >> 3) & 0xF
        man = b & 0x7
        if exp == 0xF and man == 0x7:
            tab[b] = np.nan
        elif exp == 0:
            tab[b] = sign * (man / 8.0) * 2.0 ** (-6)
        else:
            tab[b] = sign * (1.0 + man / 8.0) * 2.0 ** (exp - 7)
    return tab


E4M3 = _e4m3_table()


def fp8_bytes(t) -> np.ndarray:
    """Raw bytes of a float8_e4m3fn tensor (torch) or a uint8 array."""
    if isinstance(t, np.ndarray):
        return t.view(np.uint8)
    return t.contiguous().view(__import__("torch").uint8).cpu().numpy()


def to_np(t) -> np.ndarray:
    if isinstance(t, np.ndarray):
        return t
    import torch
    t = t.detach().cpu()
    if t.dtype == torch.bfloat16:
        return t.float().numpy()
    return t.numpy()


# ---------------------------------------------------------------- dequantisation
def dequant_hidden(hq: np.ndarray, hs: np.ndarray) -> np.ndarray:
    """Reference step "1) FP8 block-scale dequantization", hidden_states part:
    A[t, k] = fp8[t, k] * scale[k // 128, t] (scale is stored [H/128, T])."""
    T = hq.shape[0]
    a = E4M3[hq].reshape(T, H // BLOCK, BLOCK)
    return (a * hs.T.astype(np.float32)[:, :, None]).reshape(T, H)


def dequant_block(wq: np.ndarray, ws: np.ndarray) -> np.ndarray:
    """Reference step 1, weight part: W[n, k] = fp8[n, k] * S[n // 128, k // 128]."""
    N, K = wq.shape
    w = E4M3[wq].reshape(N // BLOCK, BLOCK, K // BLOCK, BLOCK)
    return (w * ws.astype(np.float32)[:, None, :, None]).reshape(N, K)


def e4m3_round(v: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest e4m3fn byte (ties to even), saturating at +-448."""
    v = np.asarray(v, np.float32)
    finite = E4M3[:127].astype(np.float64)            # bytes 0..126: 0 .. 448, ascending
    a = np.minimum(np.abs(v).astype(np.float64), 448.0)
    hi = np.searchsorted(finite, a, side="left").clip(0, 126)
    lo = (hi - 1).clip(0, 126)
    dlo, dhi = a - finite[lo], finite[hi] - a
    pick_hi = (dhi < dlo) | ((dhi == dlo) & (hi % 2 == 0))
    b = np.where(pick_hi, hi, lo).astype(np.uint8)
    b = np.where(a == finite[hi], hi, b).astype(np.uint8)
    return np.where(np.signbit(v), b | 0x80, b).astype(np.uint8)   # sign kept, -0 included


def quantize_rows(x: np.ndarray):
    """x [T, K] -> (e4m3 bytes [T, K], scales f32 [K/128, T]); s = max(amax, 1e-12)/448, q = e4m3(x/s).
    The activation layout of `...json:81-88` (scales token-contiguous)."""
    x = np.asarray(x, np.float32)
    T, K = x.shape
    xb = x.reshape(T, K // BLOCK, BLOCK)
    s = (np.maximum(np.abs(xb).max(axis=2), np.float32(1e-12)) / np.float32(448.0)).astype(np.float32)
    q = e4m3_round((xb / s[:, :, None]).astype(np.float32)).reshape(T, K)
    return q, s.T.copy()


# ---------------------------------------------------------------- routing
def route(logits: np.ndarray, bias: np.ndarray, routed_scaling_factor: float):
    """Reference step "2) No-aux routing".

    s = 1/(1+exp(-x)); sb = s + bias; group score = sum of the two largest sb in
    each of the 8 groups of 32; keep the 4 best groups; top-8 experts of sb over
    the kept groups; weight = s / (sum of the 8 s + 1e-20) * scaling factor.

    Exact ties are broken towards the lower index (torch leaves tie order
    unspecified; the tests compare selections with tie awareness).
    Returns (topk_idx int32 [T, 8] in selection order, weights f32 [T, 8]).
    """
    x = logits.astype(np.float32)
    T = x.shape[0]
    s = (np.float32(1.0) / (np.float32(1.0) + np.exp(-x))).astype(np.float32)
    sb = (s + bias.astype(np.float32)[None, :]).astype(np.float32)
    g = sb.reshape(T, N_GROUP, E_GLOBAL // N_GROUP)
    top2 = -np.sort(-g, axis=2, kind="stable")[:, :, :2]
    gscore = (top2[:, :, 0] + top2[:, :, 1]).astype(np.float32)
    # group rank: strictly larger scores, then equal scores with lower index
    gi = np.arange(N_GROUP)
    better = (gscore[:, None, :] > gscore[:, :, None]) | (
        (gscore[:, None, :] == gscore[:, :, None]) & (gi[None, None, :] < gi[None, :, None]))
    keep = better.sum(axis=2) < TOPK_GROUP                      # [T, 8]
    mask = np.repeat(keep, E_GLOBAL // N_GROUP, axis=1)
    pruned = np.where(mask, sb, -np.inf).astype(np.float32)
    # stable descending sort keeps lower index first among equal values
    order = np.argsort(-pruned, axis=1, kind="stable")[:, :TOP_K].astype(np.int32)
    sel = np.take_along_axis(s, order, axis=1)
    denom = (sel.sum(axis=1, dtype=np.float32) + np.float32(1e-20)).astype(np.float32)
    w = ((sel / denom[:, None]).astype(np.float32) * np.float32(routed_scaling_factor)).astype(np.float32)
    return order, w


# ---------------------------------------------------------------- whole operator
def moe_forward(routing_logits, routing_bias, hidden_states, hidden_states_scale,
                gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale,
                local_expert_offset: int, routed_scaling_factor: float,
                out_dtype: str = "bf16", routing=None, dequant_all: bool = False):
    """Reference step "3) Local expert compute and accumulation".

    For every local expert that some token selected: G1 = A_e W13_e^T,
    C = silu(G1[:, I:]) * G1[:, :I], O = C W2_e^T, output[tok] += w * O, all in
    fp32; the result is rounded to bf16 once (`out_dtype="f32"` skips that
    rounding, for summing expert-parallel shards).
    Inputs may be torch tensors (any device) or numpy arrays (fp8 as uint8).
    Returns a float32 numpy array (bf16-rounded values unless out_dtype="f32").
    """
    logits = to_np(routing_logits).astype(np.float32)
    bias = np.zeros(E_GLOBAL, np.float32) if routing_bias is None else to_np(routing_bias).astype(np.float32)
    T = logits.shape[0]
    E_local = gemm1_weights.shape[0]
    hq = fp8_bytes(hidden_states)
    hs = to_np(hidden_states_scale).astype(np.float32)
    if routing is None:
        topk_idx, w = route(logits, bias, routed_scaling_factor)
    else:
        topk_idx, w = routing
    A = dequant_hidden(hq, hs) if T else np.zeros((0, H), np.float32)
    out = np.zeros((T, H), np.float32)
    off = int(local_expert_offset)
    deq = None
    if dequant_all:   # the reference's order: every local expert's weights first (step 1)
        deq = [(dequant_block(fp8_bytes(gemm1_weights[le]), to_np(gemm1_weights_scale[le])),
                dequant_block(fp8_bytes(gemm2_weights[le]), to_np(gemm2_weights_scale[le])))
               for le in range(E_local)]
    for le in range(E_local):
        ge = off + le
        if ge < 0 or ge >= E_GLOBAL:
            continue
        hit = topk_idx == ge
        rows = np.nonzero(hit.any(axis=1))[0]
        if rows.size == 0:
            continue
        if deq is not None:
            w13, w2 = deq[le]
        else:
            w13 = dequant_block(fp8_bytes(gemm1_weights[le]), to_np(gemm1_weights_scale[le]))
            w2 = dequant_block(fp8_bytes(gemm2_weights[le]), to_np(gemm2_weights_scale[le]))
        g1 = A[rows] @ w13.T
        x1, x2 = g1[:, :I], g1[:, I:]
        c = (x2 / (np.float32(1.0) + np.exp(-x2))) * x1
        o = c @ w2.T
        wt = (w * hit)[rows].sum(axis=1).astype(np.float32)
        out[rows] += o * wt[:, None]
    if out_dtype == "f32":
        return out
    return bf16_round(out)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even), kept as float32."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    r = r.astype(np.uint32)
    nan = np.isnan(x)
    out = r.view(np.float32).copy()
    out[nan] = np.nan
    return out


def local_pairs(topk_idx: np.ndarray, local_expert_offset: int, num_local_experts: int) -> int:
    """Number of (token, local expert) pairs: the rows the grouped GEMMs process."""
    le = topk_idx - int(local_expert_offset)
    return int(((le >= 0) & (le < num_local_experts)).sum())


def hit_experts(topk_idx: np.ndarray, local_expert_offset: int, num_local_experts: int) -> int:
    le = topk_idx - int(local_expert_offset)
    le = le[(le >= 0) & (le < num_local_experts)]
    return int(np.unique(le).size)
