"""CPU (gloo, 2 and 4 ranks): the host side of the peer-memory expert-parallel
transport (ep.PeerExpertParallel).

Each rank is a process. The CUDA kernels are replaced by a numpy stand-in that
keeps the kernels' buffer layout and flag protocol: the exchange buffer is a
set of files mapped by every rank (np.memmap; the "IPC handle" is the file
prefix, exchanged over gloo exactly like the CUDA handle), dispatch writes the
selections of every token slot to every rank at row (source, slot) and the
token's row to the ranks owning one of its experts, then raises the
destination's dispatch flag to the step's epoch; waits spin (bounded) on the
flags other processes write; the return writes fp32 rows to [rank][slot] of
the source's buffer; combine sums them in ascending rank order.

The stand-in operator is additive over experts, partial[t] = sum over the
rank's experts among t's picks of w * (e + 1) * (1 + mean of t's FP8 bytes), so
every token's combined row has a closed form. Three steps with changing ragged
token counts check that stale rows of an earlier step never leak.
"""
import os
import socket
import tempfile
import time

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import __graft_entry__ as ge

H = 7168


class NumpyPeerBackend:
    """Host stand-in for LibraryPeerBackend with the same layouts and protocol."""

    def __init__(self, oracle, root):
        self.O = oracle
        self.root = root
        self.n = 0

    def _arrays(self, prefix, C, W, mode):
        N = C * W
        spec = {"flags": (np.int64, (2, W)), "idx": (np.int32, (N, 8)), "w": (np.float32, (N, 8)),
                "hidden": (np.uint8, (N, H)), "scale": (np.float32, (56, N)), "ret": (np.float32, (N, H))}
        return {k: np.memmap(f"{prefix}.{k}", dtype=dt, mode=mode, shape=sh) for k, (dt, sh) in spec.items()}

    # buffers: `base` is the file prefix (a str); handles are its bytes
    def alloc(self, capacity, world):
        self.n += 1
        prefix = os.path.join(self.root, f"r{os.getpid()}_{self.n}")
        a = self._arrays(prefix, capacity, world, "w+")
        for v in a.values():
            v.flush()
        return prefix

    def free(self, base):
        pass

    def handle(self, base):
        return base.encode()

    def open(self, handle):
        return handle.decode()

    def close(self, base):
        pass

    def peer_table(self, bases):
        return list(bases)

    def _peer(self, st, d):
        return self._arrays(st.peer_bases[d], st.capacity, st.world, "r+")

    # one step
    def route(self, st, logits, bias, scale):
        idx, w = self.O.route(logits.numpy(), bias.float().numpy(), scale)
        st.topk_idx, st.topk_w = idx.astype(np.int32), w.astype(np.float32)

    def dispatch(self, st, hidden, hs, T):
        C, W, r, epr = st.capacity, st.world, st.rank, st.epr
        hb = hidden.view(torch.uint8).numpy() if T else np.zeros((0, H), np.uint8)
        hsn = hs.numpy()
        for d in range(W):
            P = self._peer(st, d)
            rows = r * C + np.arange(C)
            ids = np.full((C, 8), -1, np.int32)
            ws = np.zeros((C, 8), np.float32)
            ids[:T], ws[:T] = st.topk_idx, st.topk_w
            P["idx"][rows], P["w"][rows] = ids, ws
            to_d = np.nonzero(((st.topk_idx // epr) == d).any(1))[0] if T else np.zeros(0, int)
            P["hidden"][r * C + to_d] = hb[to_d]
            P["scale"][:, r * C + to_d] = hsn[:, to_d]
            for v in P.values():
                v.flush()
            P["flags"][0, r] = st.epoch
            P["flags"].flush()

    def wait(self, st, which):
        F = self._arrays(st.base, st.capacity, st.world, "r")["flags"]
        t0 = time.time()
        while (np.asarray(F[which]) < st.epoch).any():
            if time.time() - t0 > 60:
                raise TimeoutError("peer flag wait ran out")
            time.sleep(0.002)
            F = self._arrays(st.base, st.capacity, st.world, "r")["flags"]

    def compute(self, st, w13, s13, w2, s2, scale):
        A = self._arrays(st.base, st.capacity, st.world, "r")
        lo = st.rank * st.epr
        idx, w = np.asarray(A["idx"]), np.asarray(A["w"])
        loc = (idx >= lo) & (idx < lo + st.epr)
        mean = np.asarray(A["hidden"]).astype(np.float64).mean(1)
        st.partial = ((w * (idx + 1) * loc).sum(1) * (1.0 + mean)).astype(np.float32)
        st.has_local = loc.any(1)

    def give_back(self, st):
        C, W, r = st.capacity, st.world, st.rank
        for s in range(W):
            rows = np.nonzero(st.has_local[s * C:(s + 1) * C])[0]
            P = self._peer(st, s)
            P["ret"][r * C + rows] = st.partial[s * C + rows][:, None]
            P["ret"].flush()
            P["flags"][1, r] = st.epoch
            P["flags"].flush()

    def combine(self, st, out, T):
        A = self._arrays(st.base, st.capacity, st.world, "r")
        acc = np.zeros((T, H), np.float32)
        for d in range(st.world):
            m = ((st.topk_idx // st.epr) == d).any(1) if T else np.zeros(0, bool)
            acc[m] += np.asarray(A["ret"][d * st.capacity + np.arange(T)])[m]
        out.copy_(torch.from_numpy(acc).to(torch.bfloat16))

    def read_error(self, st):
        return 0


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, root, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ge.load_package()
        import fused_moe_b200.ep as ep
        O = ge.load_oracle()
        C = 24
        peer = ep.PeerExpertParallel(rank, world, C, backend=NumpyPeerBackend(O, root))
        gb = torch.Generator().manual_seed(5)
        bias = (torch.randn(256, generator=gb) * 0.1).to(torch.bfloat16)
        epr = 256 // world
        ok, worst = True, 0.0
        for step in range(3):
            T = [C, 7 + 5 * rank, 3 if rank % 2 else 0][step]       # ragged, shrinking, empty
            g = torch.Generator().manual_seed(1000 * step + rank)
            logits = torch.randn(T, 256, generator=g)
            hidden = torch.randint(0, 120, (T, H), generator=g, dtype=torch.uint8).view(torch.float8_e4m3fn)
            hs = torch.rand(56, T, generator=g)
            w13 = torch.zeros(epr, 1, 1)
            out = peer.forward(logits, bias, hidden, hs, w13, None, None, None, 2.5,
                               output=torch.empty(T, H, dtype=torch.bfloat16))
            idx, w = O.route(logits.numpy(), bias.float().numpy(), 2.5)
            want = (w * (idx + 1)).sum(1) * (1.0 + hidden.view(torch.uint8).float().mean(1).numpy())
            got = out.float()[:, 0].numpy()
            if T:
                worst = max(worst, float(np.abs(got - want).max()))
                ok &= bool(np.allclose(got, want, rtol=1e-2, atol=1e-2))
                ok &= bool((out.float() == out.float()[:, :1]).all())
            ok &= peer.epoch == step + 1
        result_q.put((rank, ok, worst))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_peer_transport_host_protocol_gloo(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    with tempfile.TemporaryDirectory() as root:
        procs = [ctx.Process(target=_worker, args=(r, world, port, root, q)) for r in range(world)]
        for p in procs:
            p.start()
        results = sorted(q.get(timeout=300) for _ in range(world))
        for p in procs:
            p.join(timeout=60)
            assert p.exitcode == 0
    for rank, ok, err in results:
        assert ok, f"rank {rank}: max err {err}"
