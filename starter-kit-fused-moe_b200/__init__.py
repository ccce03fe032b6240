"""B200 (sm_100a) DeepSeek-V3 FP8 block-scale fused MoE: host side.

`run(...)` keeps the reference entry point's signature and behaviour
(solution/triton/current_kernel.py:1912-2050; C++ form solution/cuda/main.cpp:38-117):
ten inputs plus an optional pre-allocated bf16 `output` (destination-passing
style); without `output` the result is returned. CPU inputs are moved to the
current CUDA device, as the reference does (current_kernel.py:1938-1956).
Shape errors raise ValueError, a missing GPU raises RuntimeError.

Everything is computed by the hand-written sm_100a kernels of `libmoe_b200.so`
through its C ABI (`include/moe_fp8.h`); there is no CPU fallback: if the
library is missing, every call raises.
"""
from __future__ import annotations

import ctypes
import pathlib
import threading

import torch

from . import inputs  # noqa: F401  (seeded synthetic inputs, re-exported)

HERE = pathlib.Path(__file__).resolve().parent
LIB_PATH = HERE / "libmoe_b200.so"

H = 7168
I = 2048
E_GLOBAL = 256
TOP_K = 8

MOE_OK = 0
_ERRORS = {1: ValueError, 2: RuntimeError, 3: RuntimeError, 4: RuntimeError}


class MoeFp8Args(ctypes.Structure):
    _fields_ = [
        ("routing_logits", ctypes.c_void_p),
        ("routing_bias", ctypes.c_void_p),
        ("hidden_states", ctypes.c_void_p),
        ("hidden_states_scale", ctypes.c_void_p),
        ("gemm1_weights", ctypes.c_void_p),
        ("gemm1_weights_scale", ctypes.c_void_p),
        ("gemm2_weights", ctypes.c_void_p),
        ("gemm2_weights_scale", ctypes.c_void_p),
        ("local_expert_offset", ctypes.c_int32),
        ("routed_scaling_factor", ctypes.c_float),
        ("output", ctypes.c_void_p),
        ("num_tokens", ctypes.c_int32),
        ("num_local_experts", ctypes.c_int32),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_size_t),
    ]


class MoeFp8WorkspaceView(ctypes.Structure):
    _fields_ = [
        ("topk_idx", ctypes.c_void_p),
        ("topk_weights", ctypes.c_void_p),
        ("expert_counts", ctypes.c_void_p),
        ("device_error", ctypes.c_void_p),
        ("pair_capacity", ctypes.c_int32),
    ]


EXPORTED_SYMBOLS = (
    "moe_fp8_block_scale_run", "moe_fp8_workspace_bytes", "moe_fp8_route", "moe_fp8_workspace_view",
    "moe_fp8_read_device_error", "moe_fp8_last_error", "moe_fp8_kernels_per_call", "moe_fp8_run_stage",
    "moe_fp8_set_gemm_path", "moe_fp8_gemm_path", "moe_fp8_route_static",
    "moe_fp8_ep_plan", "moe_fp8_ep_pack", "moe_fp8_ep_scales", "moe_fp8_ep_combine",
    "moe_fp8_quantize_activations", "moe_fp8_set_deterministic", "moe_fp8_debug_set_waits", "moe_fp8_set_cta_pair",
    "moe_fp8_block_scale_run_routed", "moe_fp8_ep_peer_buffer_bytes", "moe_fp8_ep_peer_buffer_alloc",
    "moe_fp8_ep_peer_buffer_free", "moe_fp8_ep_peer_ipc_handle", "moe_fp8_ep_peer_ipc_open",
    "moe_fp8_ep_peer_ipc_close", "moe_fp8_ep_peer_recv_view", "moe_fp8_ep_peer_dispatch", "moe_fp8_ep_peer_wait",
    "moe_fp8_ep_peer_return", "moe_fp8_ep_peer_combine", "moe_fp8_ep_peer_read_error",
)

_lib = None
_lib_lock = threading.Lock()


def load_library(path: str | pathlib.Path | None = None) -> ctypes.CDLL:
    """Load libmoe_b200.so (built by build.py) and declare its C signatures."""
    global _lib
    with _lib_lock:
        if _lib is not None and path is None:
            return _lib
        p = pathlib.Path(path) if path else LIB_PATH
        if not p.exists():
            raise RuntimeError(f"{p.name} is not built; run `python starter-kit-fused-moe_b200/build.py`")
        lib = ctypes.CDLL(str(p))
        vp, i32, sz = ctypes.c_void_p, ctypes.c_int32, ctypes.c_size_t
        lib.moe_fp8_block_scale_run.argtypes = [ctypes.POINTER(MoeFp8Args), vp]
        lib.moe_fp8_block_scale_run.restype = ctypes.c_int
        lib.moe_fp8_run_stage.argtypes = [ctypes.POINTER(MoeFp8Args), i32, vp]
        lib.moe_fp8_run_stage.restype = ctypes.c_int
        lib.moe_fp8_workspace_bytes.argtypes = [i32, i32]
        lib.moe_fp8_workspace_bytes.restype = sz
        lib.moe_fp8_route.argtypes = [vp, vp, i32, i32, i32, ctypes.c_float, vp, sz, vp]
        lib.moe_fp8_route.restype = ctypes.c_int
        lib.moe_fp8_route_static.argtypes = [vp, vp, i32, i32, i32, ctypes.c_float, vp, vp, vp]
        lib.moe_fp8_route_static.restype = ctypes.c_int
        lib.moe_fp8_workspace_view.argtypes = [vp, i32, i32, ctypes.POINTER(MoeFp8WorkspaceView)]
        lib.moe_fp8_workspace_view.restype = ctypes.c_int
        lib.moe_fp8_read_device_error.argtypes = [vp, vp, ctypes.POINTER(i32)]
        lib.moe_fp8_read_device_error.restype = ctypes.c_int
        lib.moe_fp8_last_error.argtypes = []
        lib.moe_fp8_last_error.restype = ctypes.c_char_p
        lib.moe_fp8_set_gemm_path.argtypes = [i32]
        lib.moe_fp8_set_gemm_path.restype = i32
        lib.moe_fp8_set_cta_pair.argtypes = [i32]
        lib.moe_fp8_set_cta_pair.restype = i32
        lib.moe_fp8_set_deterministic.argtypes = [i32]
        lib.moe_fp8_set_deterministic.restype = i32
        lib.moe_fp8_gemm_path.argtypes = [i32]
        lib.moe_fp8_gemm_path.restype = i32
        lib.moe_fp8_debug_trace.argtypes = [i32, vp, i32]
        lib.moe_fp8_debug_trace.restype = ctypes.c_int
        lib.moe_fp8_debug_set_waits.argtypes = [ctypes.c_uint64, i32]
        lib.moe_fp8_debug_set_waits.restype = ctypes.c_int
        lib.moe_fp8_kernels_per_call.argtypes = [i32]
        lib.moe_fp8_kernels_per_call.restype = i32
        if path is None:
            _lib = lib
        return lib


def _check(rc: int, what: str):
    if rc != MOE_OK:
        msg = load_library().moe_fp8_last_error().decode(errors="replace")
        raise _ERRORS.get(rc, RuntimeError)(f"{what}: {msg} (status {rc})")


# ------------------------------------------------------------------ workspace cache
_ws: dict[int, torch.Tensor] = {}


def workspace(num_tokens: int, num_local_experts: int, device: torch.device) -> torch.Tensor:
    """Per-device byte buffer, grown on demand and reused across calls (the
    reference's op-owned cache, solution/cuda/kernel.cu:25-56)."""
    need = int(load_library().moe_fp8_workspace_bytes(int(num_tokens), int(num_local_experts)))
    idx = device.index if device.index is not None else torch.cuda.current_device()
    buf = _ws.get(idx)
    if buf is None or buf.numel() < need:
        _ws.pop(idx, None)
        buf = torch.zeros(max(need, 1 << 20), dtype=torch.uint8, device=torch.device("cuda", idx))
        _ws[idx] = buf
    return buf


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream_handle(device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _to_dev(t, device, dtype=None):
    if t is None:
        return None
    if dtype is not None and t.dtype != dtype:
        t = t.to(dtype)
    if t.device != device:
        t = t.to(device, non_blocking=False)
    return t.contiguous()


def _scalar(v, kind):
    if isinstance(v, torch.Tensor):
        v = v.item()
    return kind(v)


@torch.no_grad()
def run(routing_logits, routing_bias, hidden_states, hidden_states_scale, gemm1_weights,
        gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, local_expert_offset,
        routed_scaling_factor, output=None):
    """DeepSeek-V3 FP8 block-scale MoE forward (routing, GEMM1+SwiGLU, GEMM2, combine).

    Same arguments, dtypes and layouts as the reference operator; `output`
    (bf16 [T, 7168]) is written in place when given and returned.
    """
    if not torch.cuda.is_available():
        raise RuntimeError("CUDA is required: this operator has no CPU implementation")
    lib = load_library()
    dev = hidden_states.device if hidden_states.is_cuda else torch.device("cuda", torch.cuda.current_device())
    if routing_logits.dim() != 2 or routing_logits.shape[1] != E_GLOBAL:
        raise ValueError(f"routing_logits must be [T, {E_GLOBAL}], got {tuple(routing_logits.shape)}")
    T = int(routing_logits.shape[0])
    E = int(gemm1_weights.shape[0])
    exp = {
        "hidden_states": (hidden_states, (T, H)),
        "hidden_states_scale": (hidden_states_scale, (H // 128, T)),
        "gemm1_weights": (gemm1_weights, (E, 2 * I, H)),
        "gemm1_weights_scale": (gemm1_weights_scale, (E, 2 * I // 128, H // 128)),
        "gemm2_weights": (gemm2_weights, (E, H, I)),
        "gemm2_weights_scale": (gemm2_weights_scale, (E, H // 128, I // 128)),
    }
    for name, (t, shape) in exp.items():
        if tuple(t.shape) != shape:
            raise ValueError(f"{name} must have shape {shape}, got {tuple(t.shape)}")
    for name in ("hidden_states", "gemm1_weights", "gemm2_weights"):
        if exp[name][0].dtype != torch.float8_e4m3fn:
            raise ValueError(f"{name} must be float8_e4m3fn, got {exp[name][0].dtype}")
    if routing_bias is not None and routing_bias.shape[-1] != E_GLOBAL:
        raise ValueError(f"routing_bias must have {E_GLOBAL} entries")
    if not 1 <= E <= 256:
        raise ValueError("number of local experts must be in [1, 256]")
    offset = _scalar(local_expert_offset, int)
    scale = _scalar(routed_scaling_factor, float)

    logits = _to_dev(routing_logits, dev, torch.float32)
    bias = _to_dev(routing_bias.reshape(-1), dev, torch.bfloat16) if routing_bias is not None else None
    hq = _to_dev(hidden_states, dev)
    hs = _to_dev(hidden_states_scale, dev, torch.float32)
    w13 = _to_dev(gemm1_weights, dev)
    s13 = _to_dev(gemm1_weights_scale, dev, torch.float32)
    w2 = _to_dev(gemm2_weights, dev)
    s2 = _to_dev(gemm2_weights_scale, dev, torch.float32)

    if output is None:
        out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
    else:
        if tuple(output.shape) != (T, H) or output.dtype != torch.bfloat16:
            raise ValueError(f"output must be bfloat16 [{T}, {H}], got {output.dtype} {tuple(output.shape)}")
        out = output if (output.is_cuda and output.is_contiguous() and output.device == dev) else \
            torch.empty(T, H, dtype=torch.bfloat16, device=dev)
    if T > 0:
        with torch.cuda.device(dev):
            ws = workspace(T, E, dev)
            a = MoeFp8Args(
                _ptr(logits), _ptr(bias), _ptr(hq), _ptr(hs), _ptr(w13), _ptr(s13), _ptr(w2), _ptr(s2),
                offset, scale, _ptr(out), T, E, _ptr(ws), ws.numel())
            _check(lib.moe_fp8_block_scale_run(ctypes.byref(a), _stream_handle(dev)), "moe_fp8_block_scale_run")
    if output is not None and out is not output:
        output.copy_(out)
        return output
    return out


@torch.no_grad()
def route(routing_logits, routing_bias, local_expert_offset=0, num_local_experts=32,
          routed_scaling_factor=2.5):
    """Routing kernel alone. Returns (topk_idx int32 [T, 8], topk_weights f32 [T, 8],
    expert_counts int32 [E]) as CUDA tensors (copies out of the workspace)."""
    lib = load_library()
    dev = routing_logits.device if routing_logits.is_cuda else torch.device("cuda", torch.cuda.current_device())
    T = int(routing_logits.shape[0])
    E = int(num_local_experts)
    logits = _to_dev(routing_logits, dev, torch.float32)
    bias = _to_dev(routing_bias.reshape(-1), dev, torch.bfloat16) if routing_bias is not None else None
    with torch.cuda.device(dev):
        ws = workspace(T, E, dev)
        _check(lib.moe_fp8_route(_ptr(logits), _ptr(bias), T, int(local_expert_offset), E,
                                 float(routed_scaling_factor), _ptr(ws), ws.numel(), _stream_handle(dev)),
               "moe_fp8_route")
        return workspace_tensors(ws, T, E)


def workspace_tensors(ws: torch.Tensor, T: int, E: int):
    """Copies of (topk_idx, topk_weights, expert_counts) held in a workspace."""
    lib = load_library()
    v = MoeFp8WorkspaceView()
    _check(lib.moe_fp8_workspace_view(_ptr(ws), T, E, ctypes.byref(v)), "moe_fp8_workspace_view")
    base = ws.data_ptr()

    def view(addr, n, dtype):
        off = addr - base
        nbytes = n * torch.tensor([], dtype=dtype).element_size()
        return ws[off:off + nbytes].view(dtype).clone()

    return (view(v.topk_idx, T * TOP_K, torch.int32).view(T, TOP_K),
            view(v.topk_weights, T * TOP_K, torch.float32).view(T, TOP_K),
            view(v.expert_counts, E, torch.int32))


GEMM_PATHS = {0: "tile kernels", 1: "streaming GEMM1 + tile GEMM2", 2: "fused streaming GEMM1+GEMM2",
              3: "streaming GEMM1 + streaming GEMM2"}


@torch.no_grad()
def quantize_activations(x):
    """bf16 / f32 [T, 7168] CUDA tensor -> (e4m3 [T, 7168], f32 scales [56, T]), the operator's input layout."""
    lib = load_library()
    if x.dim() != 2 or x.shape[1] != H or x.dtype not in (torch.bfloat16, torch.float32):
        raise ValueError("x must be bf16 or f32 [T, 7168]")
    x = x.contiguous()
    T = int(x.shape[0])
    q = torch.empty(T, H, dtype=torch.float8_e4m3fn, device=x.device)
    s = torch.empty(H // 128, T, dtype=torch.float32, device=x.device)
    lib.moe_fp8_quantize_activations.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p,
                                                 ctypes.c_void_p, ctypes.c_void_p]
    with torch.cuda.device(x.device):
        _check(lib.moe_fp8_quantize_activations(_ptr(x), int(x.dtype == torch.bfloat16), T, _ptr(q), _ptr(s),
                                                _stream_handle(x.device)), "moe_fp8_quantize_activations")
    return q, s


def set_deterministic(on: bool) -> bool:
    """Bit-reproducible combine (see moe_fp8_set_deterministic); returns the previous setting.
    Workspaces obtained before the switch are re-sized on the next call."""
    return bool(load_library().moe_fp8_set_deterministic(1 if on else 0))


def set_gemm_path(path: int) -> int:
    """Force a GEMM kernel family (0..3, see GEMM_PATHS) or -1 for automatic; returns the previous setting."""
    return int(load_library().moe_fp8_set_gemm_path(int(path)))


def set_cta_pair(on: bool) -> bool:
    """Run the tile GEMMs as two-CTA clusters (see moe_fp8_set_cta_pair); returns the previous setting."""
    return bool(load_library().moe_fp8_set_cta_pair(1 if on else 0))


def gemm_path(num_tokens: int) -> int:
    """GEMM kernel family a call with `num_tokens` tokens uses."""
    return int(load_library().moe_fp8_gemm_path(int(num_tokens)))


def read_device_error(device=None) -> int:
    """Read and clear the kernels' sticky error bits for `device` (0 = none)."""
    lib = load_library()
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else torch.device(device).index)
    ws = _ws.get(dev.index)
    if ws is None:
        return 0
    bits = ctypes.c_int32(0)
    with torch.cuda.device(dev):
        rc = lib.moe_fp8_read_device_error(_ptr(ws), _stream_handle(dev), ctypes.byref(bits))
    if rc not in (MOE_OK, 4):
        _check(rc, "moe_fp8_read_device_error")
    return int(bits.value)
