"""ctypes binding of ``_kq_b200.so`` (the C ABI in ``include/kq_b200.h``).

Each wrapper takes torch tensors, checks them, and passes raw device pointers
and torch's current CUDA stream to the library.  There is no CPU fallback:
without the compiled library or a CUDA device every call raises.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "_kq_b200.so"

KQ_CB_3INST = 0
KQ_CB_MCG = 1
KQ_CB_MUL1 = 2
KQ_CB_SQG = 4

EXPORTED = (
    "kq_last_error",
    "kq_abi_version",
    "kq_build_labels",
    "kq_viterbi_workspace_bytes",
    "kq_viterbi_encode",
    "kq_quantize_tiles_sqg",
    "kq_quantize_tiles_procedural",
    "kq_pack_trellis",
    "kq_unpack_trellis_states",
    "kq_probe_hfma2",
    "kq_quantize_tiles_sqg_noalloc",
    "kq_trace_abt",
    "kq_bf16_to_f32_transposed",
    "kq_gemm_abt_tf32",
    "kq_hessian_workspace_bytes",
    "kq_accumulate_hessian",
    "kq_ldlq_step_encode",
    "kq_ldlq_chain_step",
    "kq_reconstruct_rotated",
)

KQ_CHAIN_MAX_ITEMS = 64


class ChainItem(ctypes.Structure):
    """kq_chain_item of include/kq_b200.h."""
    _fields_ = [("W", ctypes.c_void_p), ("P", ctypes.c_void_p), ("L", ctypes.c_void_p), ("err", ctypes.c_void_p),
                ("wq", ctypes.c_void_p), ("enc", ctypes.c_void_p), ("size_k", ctypes.c_int64),
                ("size_n", ctypes.c_int64), ("r0", ctypes.c_int64), ("end", ctypes.c_int64),
                ("tile_col0", ctypes.c_int64), ("n_tiles", ctypes.c_int64), ("labels", ctypes.c_void_p),
                ("K", ctypes.c_int32), ("reserved", ctypes.c_int32)]

_lib = None
_lock = threading.Lock()


class KQError(RuntimeError):
    pass


def load() -> ctypes.CDLL:
    """Load the library (no device work).  Raises if it has not been built."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise KQError(
                f"kquant_b200 CUDA library missing at {LIB_PATH}; build it with "
                "`python -m kquant_b200.build` (there is no CPU fallback)"
            )
        L = ctypes.CDLL(str(LIB_PATH))
        P, I, I64, SZ = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_size_t
        L.kq_last_error.restype = ctypes.c_char_p
        L.kq_abi_version.restype = I
        L.kq_build_labels.argtypes = [I, P, P, P]
        L.kq_viterbi_workspace_bytes.argtypes = [I, I64]
        L.kq_viterbi_workspace_bytes.restype = SZ
        L.kq_viterbi_encode.argtypes = [P, I64, I, P, I, P, P, P, SZ, P]
        L.kq_quantize_tiles_sqg.argtypes = [P, P, P, I64, P, I, I, P, SZ, P]
        L.kq_quantize_tiles_procedural.argtypes = [P, P, P, I64, I, I, I, P, SZ, P]
        L.kq_pack_trellis.argtypes = [P, I64, I, P, P]
        L.kq_unpack_trellis_states.argtypes = [P, I64, I, P, P]
        L.kq_probe_hfma2.argtypes = [P, I, I, I, P]
        L.kq_quantize_tiles_sqg_noalloc.argtypes = [P, P, P, I64, P, I, I, P]
        L.kq_trace_abt.argtypes = [P, P, P, I64, I64, I64, I64, P, P, P]
        L.kq_bf16_to_f32_transposed.argtypes = [P, I64, I64, I64, P, P, P]
        L.kq_gemm_abt_tf32.argtypes = [P, P, P, I64, I64, I64, I64, ctypes.c_float, ctypes.c_float, P, P]
        L.kq_ldlq_step_encode.argtypes = [P, P, I64, I64, I64, I64, I, P, I, P, P, P, I, P, SZ, P]
        L.kq_ldlq_chain_step.argtypes = [P, I, I, I, P, SZ, P]
        L.kq_reconstruct_rotated.argtypes = [P, P, P, I64, I64, P, P]
        L.kq_hessian_workspace_bytes.argtypes = [I64, I64, I]
        L.kq_hessian_workspace_bytes.restype = SZ
        L.kq_accumulate_hessian.argtypes = [P, P, I64, I64, I64, P, I64, I, P, SZ, P, P]
        for name in EXPORTED:
            f = getattr(L, name)
            if name not in ("kq_last_error", "kq_viterbi_workspace_bytes", "kq_hessian_workspace_bytes") and f.restype is ctypes.c_int:
                f.restype = I
        _lib = L
        return L


def _check(rc: int, what: str) -> None:
    if rc != 0:
        msg = load().kq_last_error().decode(errors="replace")
        raise KQError(f"{what} failed with status {rc}: {msg}")


def _stream(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _cuda(t: torch.Tensor, name: str, dtype: torch.dtype) -> None:
    if not t.is_cuda:
        raise KQError(f"{name} must be a CUDA tensor (kquant_b200 has no CPU path)")
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


# Launch accounting for the benchmark: counts every kernel this library
# launches and, when enabled, times each Viterbi launch with CUDA events on
# its stream (algorithmic work = (2C + 256) * 65,536 relaxations per tile).
class _Stats:
    def __init__(self):
        self.launches = 0
        self.timing = False
        self.events: list = []

    def reset(self, timing: bool = False):
        self.launches = 0
        self.timing = timing
        self.events = []
        self.base = None
        if timing and torch.cuda.is_available():
            self.base = torch.cuda.Event(enable_timing=True)
            self.base.record()

    def viterbi_summary(self):
        """(launches, busy seconds, total tiles, total relaxations, summed launch seconds) of timed Viterbi launches.

        Launches on concurrent streams overlap, so the busy time is the length of
        the union of their [start, end] intervals (the summed durations count the
        overlap twice).
        """
        total_s, tiles, relax = 0.0, 0, 0
        spans = []
        for a, b, n, c in self.events:
            b.synchronize()
            total_s += a.elapsed_time(b) / 1e3
            if self.base is not None:
                spans.append((self.base.elapsed_time(a), self.base.elapsed_time(b)))
            tiles += n
            relax += n * (2 * c + 256) * 65536
        busy = total_s
        if spans:
            busy, cur_a, cur_b = 0.0, None, None
            for a, b in sorted(spans):
                if cur_b is None or a > cur_b:
                    if cur_b is not None:
                        busy += cur_b - cur_a
                    cur_a, cur_b = a, b
                else:
                    cur_b = max(cur_b, b)
            busy = (busy + cur_b - cur_a) / 1e3
        return len(self.events), busy, tiles, relax, total_s


stats = _Stats()


# Workspace: one growing uint8 buffer per (device, stream), reused across
# calls on that stream (calls on one stream are ordered, so reuse is safe;
# concurrent streams get their own buffers).
_workspaces: dict[tuple[int, int], torch.Tensor] = {}


def workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    key = (idx, torch.cuda.current_stream(idx).cuda_stream)
    ws = _workspaces.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _workspaces[key] = ws
    return ws


def viterbi_workspace_bytes(K: int, n_tiles: int) -> int:
    return int(load().kq_viterbi_workspace_bytes(int(K), int(n_tiles)))


def build_labels(kind: int, lut: torch.Tensor | None, device: torch.device) -> torch.Tensor:
    """65,536 binary16 labels (as int16 bits) of a codebook, on ``device``."""
    out = torch.empty(65536, dtype=torch.int16, device=device)
    lp = None
    if kind == KQ_CB_SQG:
        if lut is None:
            raise ValueError("SQG labels need a LUT")
        _cuda(lut, "lut", torch.uint8)
        if lut.numel() != 65536:
            raise ValueError("codebook must contain 65,536 uint8 E4M3 values")
        lp = lut.data_ptr()
    with torch.cuda.device(device):
        _check(load().kq_build_labels(int(kind), lp, out.data_ptr(), _stream(device)), "kq_build_labels")
    stats.launches += 1
    return out


def viterbi_encode(tiles: torch.Tensor, K: int, labels: torch.Tensor, tailbite_context: int = 128,
                   out: torch.Tensor | None = None, states: torch.Tensor | None = None):
    """Encode [N, 256] fp32 tiles; returns (values fp32 [N,256], states int16 [N,256])."""
    _cuda(tiles, "tiles", torch.float32)
    _cuda(labels, "labels", torch.int16)
    if tiles.ndim != 2 or tiles.shape[1] != 256:
        raise ValueError("tiles must have shape [N, 256]")
    n = tiles.shape[0]
    dev = tiles.device
    if out is None:
        out = torch.empty_like(tiles)
    if states is None:
        states = torch.empty((n, 256), dtype=torch.int16, device=dev)
    _cuda(out, "out", torch.float32)
    _cuda(states, "states", torch.int16)
    if n == 0:
        return out, states
    with torch.cuda.device(dev):
        need = viterbi_workspace_bytes(K, n)
        if need == 0:
            raise ValueError(f"unsupported K={K}")
        ws = workspace(dev, need)
        if stats.timing:
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record()
        _check(load().kq_viterbi_encode(tiles.data_ptr(), n, int(K), labels.data_ptr(), int(tailbite_context),
                                        out.data_ptr(), states.data_ptr(), ws.data_ptr(), ws.numel(),
                                        _stream(dev)), "kq_viterbi_encode")
        if stats.timing:
            b.record()
            stats.events.append((a, b, n, int(tailbite_context)))
        stats.launches += 1
    return out, states


def pack_trellis(states: torch.Tensor, K: int) -> torch.Tensor:
    """[..., 256] int16 states -> [..., 16K] int16 words (native EXL order)."""
    _cuda(states, "states", torch.int16)
    if states.shape[-1] != 256:
        raise ValueError("states must end in a 256 dimension")
    n = states.numel() // 256
    out = torch.empty((*states.shape[:-1], 16 * K), dtype=torch.int16, device=states.device)
    with torch.cuda.device(states.device):
        _check(load().kq_pack_trellis(states.data_ptr(), n, int(K), out.data_ptr(), _stream(states.device)),
               "kq_pack_trellis")
    stats.launches += 1
    return out


def unpack_trellis_states(packed: torch.Tensor, K: int) -> torch.Tensor:
    """[..., 16K] int16 words -> [..., 256] int16 cyclic states."""
    _cuda(packed, "packed", torch.int16)
    if packed.shape[-1] != 16 * K:
        raise ValueError(f"packed tiles must end in {16 * K} int16 words")
    n = packed.numel() // (16 * K)
    out = torch.empty((*packed.shape[:-1], 256), dtype=torch.int16, device=packed.device)
    with torch.cuda.device(packed.device):
        _check(load().kq_unpack_trellis_states(packed.data_ptr(), n, int(K), out.data_ptr(),
                                               _stream(packed.device)), "kq_unpack_trellis_states")
    stats.launches += 1
    return out


def measure_hfma2_rate(device: torch.device, iters: int = 4096, reps: int = 5) -> float:
    """Measured HFMA2 instructions per second (lane-level) on ``device``."""
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    blocks, threads = sms * 4, 512
    out = torch.zeros(blocks, dtype=torch.int32, device=device)
    with torch.cuda.device(device):
        st = _stream(device)
        _check(load().kq_probe_hfma2(out.data_ptr(), 64, blocks, threads, st), "kq_probe_hfma2")
        best = float("inf")
        for _ in range(reps):
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record()
            _check(load().kq_probe_hfma2(out.data_ptr(), iters, blocks, threads, st), "kq_probe_hfma2")
            b.record()
            b.synchronize()
            best = min(best, a.elapsed_time(b) / 1e3)
    return blocks * threads * iters * 128 / best


def trace_abt_supported(M: int, N: int, Kd: int) -> bool:
    return M > 0 and N > 0 and Kd > 0 and M % 128 == 0 and N % 256 == 0 and Kd % 32 == 0


def trace_abt(A: torch.Tensor, B: torch.Tensor, D: torch.Tensor) -> torch.Tensor:
    """Device fp64 scalar sum((A @ B.T) * D) on the tensor cores (TF32 inputs, fp32 accumulate)."""
    for name, t in (("A", A), ("B", B), ("D", D)):
        _cuda(t, name, torch.float32)
    M, Kd = A.shape
    N = B.shape[0]
    if B.shape[1] != Kd or D.shape != (M, N):
        raise ValueError("trace_abt: shapes must be A [M, Kd], B [N, Kd], D [M, N]")
    out = torch.zeros((), dtype=torch.float64, device=A.device)
    err = torch.zeros((), dtype=torch.int32, device=A.device)
    with torch.cuda.device(A.device):
        _check(load().kq_trace_abt(A.data_ptr(), B.data_ptr(), D.data_ptr(), M, N, Kd, N, out.data_ptr(),
                                   err.data_ptr(), _stream(A.device)), "kq_trace_abt")
    stats.launches += 1
    _trace_errors.append(err)
    return out


_trace_errors: list = []


def check_trace_errors() -> None:
    """Raise if any tensor-core trace launch reported an internal timeout (one device sync)."""
    errs, _trace_errors[:] = list(_trace_errors), []
    if errs and int(torch.stack(errs).sum().item()):
        raise KQError("kq_trace_abt: an internal wait timed out")


def bf16_to_f32_transposed(src: torch.Tensor, row_perm: torch.Tensor | None = None) -> torch.Tensor:
    """bf16 [rows, cols] -> fp32 [cols, rows] with optional row gather: out[c, r] = src[row_perm[r], c]."""
    if not src.is_cuda or src.dtype != torch.bfloat16 or src.ndim != 2 or src.stride(1) != 1:
        raise ValueError("src must be a CUDA bf16 matrix with unit column stride")
    rows = src.shape[0] if row_perm is None else row_perm.shape[0]
    cols = src.shape[1]
    pp = None
    if row_perm is not None:
        _cuda(row_perm, "row_perm", torch.int64)
        pp = row_perm.data_ptr()
    out = torch.empty((cols, rows), dtype=torch.float32, device=src.device)
    with torch.cuda.device(src.device):
        _check(load().kq_bf16_to_f32_transposed(src.data_ptr(), rows, cols, src.stride(0), pp, out.data_ptr(),
                                                _stream(src.device)), "kq_bf16_to_f32_transposed")
    stats.launches += 1
    return out


def gemm_abt_tf32(A: torch.Tensor, B: torch.Tensor, C: torch.Tensor, alpha: float = 1.0, beta: float = 1.0) -> None:
    """C = alpha * A @ B.T + beta * C on the tensor cores (TF32 operands), in place."""
    for name, t in (("A", A), ("B", B), ("C", C)):
        _cuda(t, name, torch.float32)
    M, Kd = A.shape
    N = B.shape[0]
    if B.shape[1] != Kd or C.shape != (M, N):
        raise ValueError("gemm_abt_tf32: shapes must be A [M, Kd], B [N, Kd], C [M, N]")
    err = torch.zeros((), dtype=torch.int32, device=A.device)
    with torch.cuda.device(A.device):
        _check(load().kq_gemm_abt_tf32(A.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, Kd, N, float(alpha),
                                       float(beta), err.data_ptr(), _stream(A.device)), "kq_gemm_abt_tf32")
    stats.launches += 1
    _trace_errors.append(err)


def hessian_workspace_bytes(tokens: int, dim: int, split: int) -> int:
    return int(load().kq_hessian_workspace_bytes(int(tokens), int(dim), int(split)))


def accumulate_hessian(x: torch.Tensor, w: torch.Tensor | None, H: torch.Tensor, split: int = 3,
                       workspace: torch.Tensor | None = None) -> torch.Tensor:
    """H += x^T diag(w) x in place (x [T, d] fp32, w [T] fp32 or None, H [d, d] fp32), symmetric result.

    split=3: 3xTF32 (fp32-grade accuracy); split=1: TF32 operands.  Returns the workspace for reuse.
    """
    _cuda(x, "x", torch.float32)
    _cuda(H, "H", torch.float32)
    T, d = x.shape
    if H.shape != (d, d):
        raise ValueError("accumulate_hessian: H must be [d, d]")
    if w is not None:
        _cuda(w, "w", torch.float32)
        if w.shape != (T,):
            raise ValueError("accumulate_hessian: w must be [T]")
    need = hessian_workspace_bytes(T, d, split)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(max(need, 16), dtype=torch.uint8, device=x.device)
    err = torch.zeros((), dtype=torch.int32, device=x.device)
    with torch.cuda.device(x.device):
        _check(load().kq_accumulate_hessian(x.data_ptr(), 0 if w is None else w.data_ptr(), T, d, d, H.data_ptr(),
                                            d, int(split), workspace.data_ptr(), workspace.numel(), err.data_ptr(),
                                            _stream(x.device)), "kq_accumulate_hessian")
    stats.launches += 2
    _trace_errors.append(err)
    return workspace


def ldlq_step_encode(W: torch.Tensor, comp: torch.Tensor, r0: int, K: int, labels: torch.Tensor,
                     tailbite_context: int, wq: torch.Tensor, err: torch.Tensor, enc: torch.Tensor,
                     max_ctas: int = 0) -> None:
    """One fused LDLQ step: Viterbi of the tiles of W[:, r0:r0+16] + comp; writes wq, err and enc rows in place.

    W, wq, err [B, k, n] fp32; comp [B, 16, n] fp32; enc [B, k/16, n/16, 256] int16 (all contiguous, CUDA).
    max_ctas > 0 caps the grid (the rest of the SMs stay free for other streams).
    """
    for name, t in (("W", W), ("comp", comp), ("wq", wq), ("err", err)):
        _cuda(t, name, torch.float32)
    _cuda(enc, "enc", torch.int16)
    _cuda(labels, "labels", torch.int16)
    B, k, n = W.shape
    if comp.shape != (B, 16, n) or wq.shape != W.shape or err.shape != W.shape or enc.shape != (B, k // 16, n // 16, 256):
        raise ValueError("ldlq_step_encode: inconsistent shapes")
    dev = W.device
    with torch.cuda.device(dev):
        need = viterbi_workspace_bytes(K, B * (n // 16))
        ws = workspace(dev, need)
        if stats.timing:
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record()
        _check(load().kq_ldlq_step_encode(W.data_ptr(), comp.data_ptr(), B, k, n, int(r0), int(K), labels.data_ptr(),
                                          int(tailbite_context), wq.data_ptr(), err.data_ptr(), enc.data_ptr(),
                                          int(max_ctas), ws.data_ptr(), ws.numel(), _stream(dev)),
               "kq_ldlq_step_encode")
        if stats.timing:
            b.record()
            stats.events.append((a, b, B * (n // 16), int(tailbite_context)))
    stats.launches += 1


def ldlq_chain_step(items, tailbite_context: int, device: torch.device, max_ctas: int = 0) -> None:
    """One launch of LDLQ chain steps; ``items`` is a sequence of ChainItem (at most KQ_CHAIN_MAX_ITEMS), each
    with its own K and label table (items of different K: one wave, even item starts)."""
    n = len(items)
    if not 1 <= n <= KQ_CHAIN_MAX_ITEMS:
        raise ValueError(f"ldlq_chain_step: 1..{KQ_CHAIN_MAX_ITEMS} items")
    arr = (ChainItem * n)(*items)
    tiles = sum(int(it.n_tiles) for it in items)
    with torch.cuda.device(device):
        need = viterbi_workspace_bytes(3, tiles)
        ws = workspace(device, need)
        if stats.timing:
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record()
        _check(load().kq_ldlq_chain_step(ctypes.cast(arr, ctypes.c_void_p), n, int(tailbite_context), int(max_ctas),
                                         ws.data_ptr(), ws.numel(), _stream(device)), "kq_ldlq_chain_step")
        if stats.timing:
            b.record()
            stats.events.append((a, b, tiles, int(tailbite_context)))
    stats.launches += 1


def reconstruct_rotated(wq: torch.Tensor, su: torch.Tensor, sv: torch.Tensor) -> torch.Tensor:
    """had_r(had_l(wq) * su) * sv with 128-blocks (row W), wq [k, n] fp32, su [k], sv [n]; a new tensor."""
    _cuda(wq, "wq", torch.float32)
    k, n = wq.shape
    su = su.reshape(-1).to(torch.float32).contiguous()
    sv = sv.reshape(-1).to(torch.float32).contiguous()
    if su.numel() != k or sv.numel() != n:
        raise ValueError("su must have k and sv n entries")
    out = torch.empty_like(wq)
    with torch.cuda.device(wq.device):
        _check(load().kq_reconstruct_rotated(wq.data_ptr(), su.data_ptr(), sv.data_ptr(), k, n, out.data_ptr(),
                                             _stream(wq.device)), "kq_reconstruct_rotated")
    stats.launches += 1
    return out
