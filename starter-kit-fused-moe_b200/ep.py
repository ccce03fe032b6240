"""Expert-parallel forward over W ranks (one process per GPU).

Two transports share the expert placement below:

* `PeerExpertParallel` (the default for CUDA tensors): every rank owns an
  exchange buffer that all peers map (CUDA IPC over NVLink / NVSwitch); the
  library's kernels write token rows and fp32 partial results straight into the
  peers' buffers and signal with (epoch) flags, so a step has no host
  synchronisation, no collective on the data path, no pack/unpack passes, and
  each token's partials are summed in fp32 and rounded once. See the
  `moe_fp8_ep_peer_*` entries of include/moe_fp8.h.
* `ep_forward` (collective transport): NCCL / gloo all-to-all of per-destination
  blocks, described next. It needs one host synchronisation per step for the
  split sizes.

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


# ---------------------------------------------------------------------------- peer-memory transport
class LibraryPeerBackend:
    """The library's peer-memory entry points (moe_fp8_ep_peer_*) and the
    operator's routed mode, called through ctypes on the current stream."""

    HANDLE_BYTES = 64

    def __init__(self, pkg):
        self.pkg = pkg
        L = self.lib = pkg.load_library()
        vp, i32, u32, sz = ctypes.c_void_p, ctypes.c_int32, ctypes.c_uint32, ctypes.c_size_t
        sig = {
            "moe_fp8_ep_peer_buffer_bytes": ([i32, i32], sz),
            "moe_fp8_ep_peer_buffer_alloc": ([i32, i32, ctypes.POINTER(vp)], ctypes.c_int),
            "moe_fp8_ep_peer_buffer_free": ([vp], ctypes.c_int),
            "moe_fp8_ep_peer_ipc_handle": ([vp, vp], ctypes.c_int),
            "moe_fp8_ep_peer_ipc_open": ([vp, ctypes.POINTER(vp)], ctypes.c_int),
            "moe_fp8_ep_peer_ipc_close": ([vp], ctypes.c_int),
            "moe_fp8_ep_peer_recv_view": ([vp, i32, i32, ctypes.POINTER(MoeFp8EpRecvView)], ctypes.c_int),
            "moe_fp8_ep_peer_dispatch": ([vp, vp, vp, vp, i32, i32, i32, i32, vp, u32, vp], ctypes.c_int),
            "moe_fp8_ep_peer_wait": ([vp, i32, i32, u32, vp], ctypes.c_int),
            "moe_fp8_ep_peer_return": ([vp, i32, i32, i32, i32, i32, vp, u32, vp], ctypes.c_int),
            "moe_fp8_ep_peer_combine": ([vp, i32, i32, i32, vp, vp, vp], ctypes.c_int),
            "moe_fp8_ep_peer_read_error": ([vp, vp, ctypes.POINTER(i32)], ctypes.c_int),
            "moe_fp8_block_scale_run_routed": ([ctypes.POINTER(pkg.MoeFp8Args), vp, vp, vp], ctypes.c_int),
        }
        for name, (args, res) in sig.items():
            f = getattr(L, name)
            f.argtypes, f.restype = args, res

    def _s(self):
        return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    def _chk(self, rc, what):
        self.pkg._check(rc, what)

    # buffers
    def alloc(self, capacity, world):
        p = ctypes.c_void_p()
        self._chk(self.lib.moe_fp8_ep_peer_buffer_alloc(capacity, world, ctypes.byref(p)), "ep buffer alloc")
        return p.value

    def free(self, base):
        self._chk(self.lib.moe_fp8_ep_peer_buffer_free(ctypes.c_void_p(base)), "ep buffer free")

    def handle(self, base):
        h = ctypes.create_string_buffer(self.HANDLE_BYTES)
        self._chk(self.lib.moe_fp8_ep_peer_ipc_handle(ctypes.c_void_p(base), h), "ep ipc handle")
        return h.raw

    def open(self, handle):
        p = ctypes.c_void_p()
        self._chk(self.lib.moe_fp8_ep_peer_ipc_open(ctypes.create_string_buffer(handle, len(handle)),
                                                    ctypes.byref(p)), "ep ipc open")
        return p.value

    def close(self, base):
        self._chk(self.lib.moe_fp8_ep_peer_ipc_close(ctypes.c_void_p(base)), "ep ipc close")

    def peer_table(self, bases):
        return (ctypes.c_void_p * len(bases))(*bases)

    # one step
    def route(self, st, logits, bias, scale):
        """Route this rank's tokens; the selections stay in st.route_ws."""
        T = int(logits.shape[0])
        p = self.pkg._ptr
        need = int(self.lib.moe_fp8_workspace_bytes(T, 1))
        if st.route_ws is None or st.route_ws.numel() < need:
            st.route_ws = torch.empty(max(need, 1 << 20), dtype=torch.uint8, device=logits.device)
        self._chk(self.lib.moe_fp8_route(p(logits), p(bias), T, 0, 1, float(scale), p(st.route_ws),
                                         st.route_ws.numel(), self._s()), "moe_fp8_route")
        v = self.pkg.MoeFp8WorkspaceView()
        self._chk(self.lib.moe_fp8_workspace_view(p(st.route_ws), T, 1, ctypes.byref(v)), "workspace view")
        st.topk_idx, st.topk_w = v.topk_idx, v.topk_weights

    def dispatch(self, st, hidden, hs, T):
        p = self.pkg._ptr
        self._chk(self.lib.moe_fp8_ep_peer_dispatch(ctypes.c_void_p(st.topk_idx), ctypes.c_void_p(st.topk_w),
                                                    p(hidden), p(hs), T, st.capacity, st.rank, st.world, st.peers,
                                                    st.epoch, self._s()), "moe_fp8_ep_peer_dispatch")

    def wait(self, st, which):
        self._chk(self.lib.moe_fp8_ep_peer_wait(ctypes.c_void_p(st.base), st.world, which, st.epoch, self._s()),
                  "moe_fp8_ep_peer_wait")

    def compute(self, st, w13, s13, w2, s2, scale):
        p = self.pkg._ptr
        N, epr = st.capacity * st.world, st.epr
        need = int(self.lib.moe_fp8_workspace_bytes(N, epr))
        if st.op_ws is None or st.op_ws.numel() < need:
            st.op_ws = torch.empty(need, dtype=torch.uint8, device=w13.device)
        rv = MoeFp8EpRecvView()
        self._chk(self.lib.moe_fp8_ep_peer_recv_view(ctypes.c_void_p(st.base), st.capacity, st.world,
                                                     ctypes.byref(rv)), "recv view")
        a = self.pkg.MoeFp8Args(None, None, ctypes.c_void_p(rv.hidden_states), ctypes.c_void_p(rv.hidden_states_scale),
                                p(w13), p(s13), p(w2), p(s2), st.rank * epr, float(scale), None, N, epr, p(st.op_ws),
                                st.op_ws.numel())
        self._chk(self.lib.moe_fp8_block_scale_run_routed(ctypes.byref(a), ctypes.c_void_p(rv.topk_idx),
                                                          ctypes.c_void_p(rv.topk_weights), self._s()),
                  "moe_fp8_block_scale_run_routed")

    def give_back(self, st):
        p = self.pkg._ptr
        self._chk(self.lib.moe_fp8_ep_peer_return(p(st.op_ws), st.epr, st.rank * st.epr, st.capacity, st.rank,
                                                  st.world, st.peers, st.epoch, self._s()), "moe_fp8_ep_peer_return")

    def combine(self, st, out, T):
        p = self.pkg._ptr
        self._chk(self.lib.moe_fp8_ep_peer_combine(ctypes.c_void_p(st.topk_idx), T, st.capacity, st.world,
                                                   ctypes.c_void_p(st.base), p(out), self._s()),
                  "moe_fp8_ep_peer_combine")

    def read_error(self, st):
        bits = ctypes.c_int32(0)
        rc = self.lib.moe_fp8_ep_peer_read_error(ctypes.c_void_p(st.base), self._s(), ctypes.byref(bits))
        if rc not in (0, 4):
            self._chk(rc, "moe_fp8_ep_peer_read_error")
        return int(bits.value)

    def pairs(self, st):
        """Local (token, expert) pairs this rank computed in its last step (host sync)."""
        _, _, counts = self.pkg.workspace_tensors(st.op_ws, st.capacity * st.world, st.epr)
        return int(counts.sum().item())


class MoeFp8EpRecvView(ctypes.Structure):
    _fields_ = [("hidden_states", ctypes.c_void_p), ("hidden_states_scale", ctypes.c_void_p),
                ("topk_idx", ctypes.c_void_p), ("topk_weights", ctypes.c_void_p), ("num_rows", ctypes.c_int32)]


class PeerExpertParallel:
    """Expert-parallel MoE over peer memory for one rank.

    Rank `rank` of `world` holds experts [rank * 256/world, (rank+1) * 256/world)
    and calls `forward` with at most `capacity` tokens per step; all ranks call
    it the same number of times (each call is one step with a new epoch). The
    exchange buffers are mapped once at construction: over `group` with CUDA IPC
    handles (one process per GPU), or, for ranks emulated in one process, from
    `peer_bases` (every rank's buffer address, shared by the caller).

    `forward` = `dispatch` (route + send), `compute` (wait, local experts on the
    received rows, send results back), `combine` (wait, sum in fp32, round); the
    three phases are separate so that ranks emulated in one process can run
    every rank's phase before any rank's next one.
    """

    def __init__(self, rank, world, capacity, group=None, peer_bases=None, backend=None, base=None):
        if E_GLOBAL % world or world > 8:
            raise ValueError("world must divide 256 and be at most 8")
        self.K = backend if backend is not None else LibraryPeerBackend(__import__(__package__ or "fused_moe_b200"))
        self.rank, self.world, self.capacity = int(rank), int(world), int(capacity)
        self.epr = E_GLOBAL // self.world
        self.epoch = 0
        self.route_ws = self.op_ws = None
        self.topk_idx = self.topk_w = None
        self._opened = []
        self.base = base if base is not None else self.K.alloc(self.capacity, self.world)
        self._own_base = base is None
        self._group = group
        self._mapped_over_group = peer_bases is None
        if peer_bases is None:
            handles = [None] * self.world
            dist.all_gather_object(handles, self.K.handle(self.base), group=group)
            bases = []
            for d in range(self.world):
                if d == self.rank:
                    bases.append(self.base)
                else:
                    b = self.K.open(handles[d])
                    self._opened.append(b)
                    bases.append(b)
        else:
            bases = list(peer_bases)
        self.peer_bases = bases
        self.peers = self.K.peer_table(bases)

    @staticmethod
    def _check_tokens(routing_logits, routing_bias, hidden_states, hidden_states_scale):
        """The kernels read these through raw pointers: shapes, dtypes and layouts must be exact."""
        T = int(routing_logits.shape[0])
        checks = ((routing_logits, (T, E_GLOBAL), torch.float32, "routing_logits"),
                  (hidden_states, (T, H), torch.float8_e4m3fn, "hidden_states"),
                  (hidden_states_scale, (H // 128, T), torch.float32, "hidden_states_scale"))
        for t, shape, dtype, name in checks:
            if tuple(t.shape) != shape or t.dtype != dtype or not t.is_contiguous():
                raise ValueError(f"{name} must be a contiguous {dtype} tensor of shape {shape}, "
                                 f"got {t.dtype} {tuple(t.shape)}")
        if routing_bias is not None and (routing_bias.numel() != E_GLOBAL or routing_bias.dtype != torch.bfloat16):
            raise ValueError("routing_bias must be bf16 with 256 entries (or None)")
        return T

    def dispatch(self, routing_logits, routing_bias, hidden_states, hidden_states_scale, routed_scaling_factor):
        T = self._check_tokens(routing_logits, routing_bias, hidden_states, hidden_states_scale)
        if T > self.capacity:
            raise ValueError(f"{T} tokens exceed the exchange capacity {self.capacity}")
        self.epoch = (self.epoch + 1) & 0xFFFFFFFF
        self.T = T
        self.K.route(self, routing_logits, routing_bias, routed_scaling_factor)
        self.K.dispatch(self, hidden_states, hidden_states_scale, T)

    def compute(self, gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, routed_scaling_factor):
        if int(gemm1_weights.shape[0]) != self.epr:
            raise ValueError(f"this rank holds {self.epr} experts, got weights for {gemm1_weights.shape[0]}")
        self.K.wait(self, 0)
        self.K.compute(self, gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale,
                       routed_scaling_factor)
        self.K.give_back(self)

    def combine(self, output=None, device=None):
        out = output if output is not None else torch.empty(self.T, H, dtype=torch.bfloat16, device=device)
        self.K.wait(self, 1)
        self.K.combine(self, out, self.T)
        return out

    @torch.no_grad()
    def forward(self, routing_logits, routing_bias, hidden_states, hidden_states_scale, gemm1_weights,
                gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, routed_scaling_factor, output=None,
                marks=None):
        """One step for this rank's tokens; returns bf16 [T, 7168]. `marks`, a
        list, receives a CUDA event after each phase (route + dispatch, compute,
        combine) for per-phase timing."""
        if int(gemm1_weights.shape[0]) != self.epr:
            raise ValueError(f"this rank holds {self.epr} experts, got weights for {gemm1_weights.shape[0]}")
        rec = (lambda: marks.append(_event())) if marks is not None else (lambda: None)
        rec()
        self.dispatch(routing_logits, routing_bias, hidden_states, hidden_states_scale, routed_scaling_factor)
        rec()
        self.K.wait(self, 0)
        rec()
        self.K.compute(self, gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale,
                       routed_scaling_factor)
        rec()
        self.K.give_back(self)
        rec()
        out = self.combine(output, device=routing_logits.device)
        rec()
        return out

    def read_error(self):
        return self.K.read_error(self)

    def close(self):
        """Unmap the peers' buffers and free this rank's. With buffers mapped
        over a process group every rank must call it (a barrier keeps a buffer
        alive until no peer can still write into it)."""
        if self._mapped_over_group and self.base is not None:
            if torch.cuda.is_available() and isinstance(self.base, int):
                torch.cuda.synchronize()
            dist.barrier(group=self._group)
        for b in self._opened:
            self.K.close(b)
        self._opened = []
        if self._own_base and self.base is not None:
            self.K.free(self.base)
        self.base = None


def _event():
    e = torch.cuda.Event(enable_timing=True)
    e.record()
    return e
