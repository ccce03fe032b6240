"""Expert-parallel forward over W ranks (one process per GPU).

Rank r holds experts [r*E/W, (r+1)*E/W) (E = 256) and the operator runs with
local_expert_offset = r*E/W, the reference's only expert-parallel hook
(`...json:146`). For its own tokens a rank:

1. routes them (same routing kernel) and plans which ranks own at least one of
   each token's 8 experts;
2. exchanges per-destination token counts, then sends each destination the
   token's routing logits, FP8 row and block scales (NCCL all-to-all);
3. runs the operator on the tokens it received, over its local experts only;
   the destination re-derives the token's routing from the logits, so the
   selection and weights are those the source computed;
4. sends each partial output row back (all-to-all in the reverse direction)
   and sums every token's partials in fp32 (combine kernel).

The data movement runs in the library's kernels (`moe_fp8_ep_*` in
include/moe_fp8.h); torch.distributed only carries the bytes. The kernel
backend is an object so the rank bookkeeping can be exercised on CPU ranks
(gloo) with a stand-in backend in the tests.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

H = 7168
E_GLOBAL = 256


class DeviceExchange:
    """The library's CUDA kernels for routing, planning, packing and combining."""

    def __init__(self, pkg):
        self.pkg = pkg
        self.lib = pkg.load_library()
        vp, i32 = ctypes.c_void_p, ctypes.c_int32
        L = self.lib
        L.moe_fp8_ep_plan.argtypes = [vp, i32, i32, i32, i32, i32, vp, vp, vp]
        L.moe_fp8_ep_pack.argtypes = [vp, vp, vp, i32, i32, vp, vp, i32, vp, vp, vp, vp]
        L.moe_fp8_ep_scales.argtypes = [vp, i32, vp, vp]
        L.moe_fp8_ep_combine.argtypes = [vp, vp, vp, i32, i32, i32, vp, vp]
        for f in (L.moe_fp8_ep_plan, L.moe_fp8_ep_pack, L.moe_fp8_ep_scales, L.moe_fp8_ep_combine):
            f.restype = ctypes.c_int

    def _s(self):
        return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    def _chk(self, rc, what):
        self.pkg._check(rc, what)

    def route(self, logits, bias, scale):
        idx, _, _ = self.pkg.route(logits, bias, 0, E_GLOBAL, scale)
        return idx

    def plan(self, topk_idx, world, experts_per_rank, wave_tokens, waves):
        T = topk_idx.shape[0]
        counts = torch.empty(waves * world, dtype=torch.int32, device=topk_idx.device)
        slot = torch.empty(T, world, dtype=torch.int32, device=topk_idx.device)
        p = self.pkg._ptr
        self._chk(self.lib.moe_fp8_ep_plan(p(topk_idx), T, world, experts_per_rank, wave_tokens, waves, p(counts),
                                           p(slot), self._s()), "moe_fp8_ep_plan")
        return counts, slot

    def pack(self, logits, hidden, hs, slot, send_off, total, wave_tokens):
        T, world = slot.shape
        dev = logits.device
        s_logits = torch.empty(total, E_GLOBAL, dtype=torch.float32, device=dev)
        s_hidden = torch.empty(total, H, dtype=torch.uint8, device=dev)
        s_scale = torch.empty(total, H // 128, dtype=torch.float32, device=dev)
        p = self.pkg._ptr
        self._chk(self.lib.moe_fp8_ep_pack(p(logits), p(hidden), p(hs), T, world, p(slot), p(send_off), wave_tokens,
                                           p(s_logits), p(s_hidden), p(s_scale), self._s()), "moe_fp8_ep_pack")
        return s_logits, s_hidden, s_scale

    def scales(self, token_major):
        N = token_major.shape[0]
        out = torch.empty(H // 128, N, dtype=torch.float32, device=token_major.device)
        p = self.pkg._ptr
        self._chk(self.lib.moe_fp8_ep_scales(p(token_major), N, p(out), self._s()), "moe_fp8_ep_scales")
        return out

    def local(self, logits, bias, hidden_u8, hs, w13, s13, w2, s2, offset, scale):
        return self.pkg.run(logits, bias, hidden_u8.view(torch.float8_e4m3fn), hs, w13, s13, w2, s2, offset, scale)

    def combine(self, back, slot, send_off, T, wave_tokens):
        world = slot.shape[1]
        out = torch.empty(T, H, dtype=torch.bfloat16, device=back.device)
        p = self.pkg._ptr
        self._chk(self.lib.moe_fp8_ep_combine(p(back), p(slot), p(send_off), wave_tokens, T, world, p(out), self._s()),
                  "moe_fp8_ep_combine")
        return out


class _Streams:
    """Compute stream = the caller's stream; communication stream = a side stream
    per device. Both collapse to no-ops for CPU tensors (gloo test ranks)."""

    _side = {}

    def __init__(self, device):
        self.cuda = device.type == "cuda"
        if self.cuda:
            self.comp = torch.cuda.current_stream(device)
            key = device.index
            if key not in self._side:
                self._side[key] = torch.cuda.Stream(device)
            self.comm = self._side[key]

    def on_comm(self):
        import contextlib
        if not self.cuda:
            return contextlib.nullcontext()
        self.comm.wait_stream(self.comp)
        return torch.cuda.stream(self.comm)


def _a2a(out, inp, out_splits, in_splits, group, async_op):
    if inp.dtype == torch.float8_e4m3fn:
        inp = inp.view(torch.uint8)
        out = out.view(torch.uint8)
    return dist.all_to_all_single(out, inp, out_splits, in_splits, group=group, async_op=async_op)


@torch.no_grad()
def ep_forward(routing_logits, routing_bias, hidden_states, hidden_states_scale, gemm1_weights,
               gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, routed_scaling_factor,
               group=None, backend=None, stats=None, waves=1):
    """Expert-parallel MoE forward for this rank's tokens; returns bf16 [T, 7168].

    The weight tensors are this rank's shard ([E/W, ...]); the rank's experts
    start at rank * E/W. All ranks of `group` must call this together with the
    same `waves` (it fixes how many collectives each rank issues; trailing waves
    may be empty). The tokens are exchanged and computed in `waves` consecutive
    groups: every wave's dispatch is issued up front on a communication stream,
    the grouped GEMMs of wave w start as soon as its tokens have arrived, and its
    partial outputs travel back while wave w + 1 computes.
    """
    K = backend if backend is not None else DeviceExchange(__import__(__package__ or "fused_moe_b200"))
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    epr = int(gemm1_weights.shape[0])
    if epr * world != E_GLOBAL:
        raise ValueError(f"{world} ranks x {epr} experts per rank must equal {E_GLOBAL}")
    T = int(routing_logits.shape[0])
    dev = routing_logits.device
    nw = int(waves)
    if nw < 1:
        raise ValueError("waves must be >= 1")
    wt = max(1, -(-T // nw))
    st = _Streams(dev)

    topk_idx = K.route(routing_logits, routing_bias, routed_scaling_factor)
    counts, slot = K.plan(topk_idx, world, epr, wt, nw)               # [nw * W], wave-major
    # every rank needs, per wave, how many tokens each peer sends it
    recv = torch.empty_like(counts)
    dist.all_to_all_single(recv, counts.view(nw, world).t().contiguous().view(-1), group=group)
    sc = counts.view(nw, world).tolist()                              # sc[w][d]: sent by me to d in wave w
    rc = recv.view(world, nw).t().tolist()                            # rc[w][s]: sent to me by s in wave w
    flat = [c for row in sc for c in row]
    off = [0]
    for c in flat[:-1]:
        off.append(off[-1] + c)
    S = sum(flat)
    send_off = torch.tensor(off, dtype=torch.int32, device=dev)
    s_logits, s_hidden, s_scale = K.pack(routing_logits, hidden_states, hidden_states_scale, slot, send_off, S, wt)

    # dispatch every wave on the communication stream
    inbox, dispatch = [], []
    with st.on_comm():
        for w in range(nw):
            lo, n_out = off[w * world], sum(sc[w])
            n_in = sum(rc[w])
            r = (torch.empty(n_in, E_GLOBAL, dtype=torch.float32, device=dev),
                 torch.empty(n_in, H, dtype=torch.uint8, device=dev),
                 torch.empty(n_in, H // 128, dtype=torch.float32, device=dev))
            works = [_a2a(r[0], s_logits[lo:lo + n_out], rc[w], sc[w], group, True),
                     _a2a(r[1], s_hidden[lo:lo + n_out], rc[w], sc[w], group, True),
                     _a2a(r[2], s_scale[lo:lo + n_out], rc[w], sc[w], group, True)]
            inbox.append(r)
            dispatch.append(works)

    back = torch.empty(S, H, dtype=torch.bfloat16, device=dev)
    returns = []
    for w in range(nw):
        for work in dispatch[w]:
            work.wait()                                               # the compute stream waits for wave w
        r_logits, r_hidden, r_scale = inbox[w]
        hs = K.scales(r_scale)
        partial = K.local(r_logits, routing_bias, r_hidden, hs, gemm1_weights, gemm1_weights_scale, gemm2_weights,
                          gemm2_weights_scale, rank * epr, routed_scaling_factor)
        lo, n_out = off[w * world], sum(sc[w])
        with st.on_comm():
            returns.append(_a2a(back[lo:lo + n_out], partial, sc[w], rc[w], group, True))
    for work in returns:
        work.wait()
    if stats is not None:
        stats.update(sent_tokens=S, received_tokens=sum(sum(r) for r in rc), waves=nw,
                     send_splits=[sum(sc[w][d] for w in range(nw)) for d in range(world)],
                     recv_splits=[sum(rc[w][s] for w in range(nw)) for s in range(world)])
    return K.combine(back, slot, send_off, T, wt)
