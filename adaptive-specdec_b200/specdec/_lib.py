"""ctypes binding of libspecdec_b200.so (declarations in include/specdec_b200.h).

The library is loaded lazily on first use.  There is no fallback: without the
built library, or with CPU tensors, every entry point raises.
"""
import ctypes
import pathlib
import threading

import torch

LIB_PATH = pathlib.Path(__file__).resolve().parent.parent / "libspecdec_b200.so"

SD_DTYPE = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}
ERRORS = {-22: "invalid argument or shape", -95: "configuration not supported",
          -28: "workspace too small", -34: "length out of range", -5: "CUDA launch failed"}

_c = ctypes
_vp, _i32, _i64, _f32, _sz = _c.c_void_p, _c.c_int, _c.c_int64, _c.c_float, _c.c_size_t

_SIGNATURES = {
    "sd_version": ([], _i32),
    "sd_sampling_workspace_bytes": ([_i32, _i32, _i32, _i32], _sz),
    "sd_verify_sample": ([_vp, _i64, _i64, _vp, _i64, _i64, _i32, _vp, _i64, _vp, _i64, _vp, _vp,
                          _i32, _i32, _i32, _f32, _f32, _i32, _vp, _vp, _vp, _vp, _vp, _sz, _vp],
                         _i32),
    "sd_verify_sample_qprobs": ([_vp, _i64, _i64, _i32, _vp, _i64, _i64, _vp, _i64, _vp, _i64, _vp,
                                 _vp, _i32, _i32, _i32, _f32, _f32, _i32, _vp, _vp, _vp, _vp, _vp,
                                 _sz, _vp], _i32),
    "sd_verify_greedy_static": ([_vp, _i64, _i64, _i32, _vp, _i64, _vp, _i64, _vp, _i32, _i32,
                                 _i32, _vp, _vp, _vp, _vp, _vp], _i32),
    "sd_draft_sample": ([_vp, _i64, _i32, _i32, _i32, _vp, _f32, _f32, _i32, _vp, _vp, _vp, _sz,
                         _vp], _i32),
    "sd_to_probs": ([_vp, _i64, _i32, _i32, _i32, _f32, _f32, _i32, _vp, _i64, _vp, _sz, _vp],
                    _i32),
    "sd_residual_probs": ([_vp, _vp, _i32, _i32, _vp, _vp], _i32),
    "sd_sample_from_probs": ([_vp, _i32, _i32, _vp, _vp, _vp], _i32),
    "sd_gather_prob": ([_vp, _i32, _i32, _vp, _vp, _vp], _i32),
    "sd_kv_lengths_update": ([_vp, _vp, _i64, _i32, _i32, _i64, _vp, _vp], _i32),
    "sd_qkv_norm_rope_append": ([_vp, _i64, _vp, _i64, _vp, _i64, _vp, _vp, _f32, _vp, _vp, _i64,
                                 _i64, _vp, _vp, _vp, _i32, _i32, _vp, _i32, _i32, _i32, _i32,
                                 _i32, _i32, _vp, _vp, _vp], _i32),
    "sd_rmsnorm": ([_vp, _i64, _vp, _f32, _vp, _i64, _i32, _i32, _vp], _i32),
    "sd_add_rmsnorm": ([_vp, _i64, _vp, _i64, _vp, _f32, _vp, _i64, _vp, _i64, _i32, _i32, _vp],
                       _i32),
    "sd_silu_mul": ([_vp, _i64, _vp, _i64, _i32, _i32, _vp], _i32),
    "sd_kv_append_paged": ([_vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp, _i32, _i32, _vp, _i32,
                            _i32, _i32, _i32, _i32, _vp, _vp], _i32),
    "sd_verify_attn_paged": ([_vp, _i64, _i64, _i64, _vp, _vp, _vp, _i32, _i32, _vp, _vp, _i32,
                              _i32, _i32, _i32, _i32, _f32, _vp, _i64, _i64, _i64, _i32, _vp,
                              _sz, _vp], _i32),
    "sd_kv_commit": ([_vp, _vp, _i32, _i32, _vp, _vp], _i32),
    "sd_kv_append": ([_vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp, _i32, _i32, _i32, _i32, _i32,
                      _i32, _vp, _vp], _i32),
    "sd_verify_attn": ([_vp, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32,
                        _i32, _f32, _vp, _i64, _i64, _i64, _i32, _vp, _sz, _vp], _i32),
    "sd_verify_attn_workspace_bytes": ([_i32, _i32, _i32, _i32, _i32, _i32], _sz),
    "sd_shard_workspace_bytes": ([_i32, _i32, _i32], _sz),
    "sd_shard_send_bytes": ([_i32, _i32, _i32, _i32, _i32], _sz),
    "sd_shard_phase": ([_vp, _i32, _vp, _vp, _vp], _i32),
}

SHARD_MAX_RANKS = 16          # SD_SHARD_MAX_RANKS
SHARD_BOUNDARY_CAP = 128      # SD_SHARD_BOUNDARY_CAP
SHARD_STATUS_FALLBACK = 2     # SD_SHARD_STATUS_FALLBACK


class ShardArgs(ctypes.Structure):
    """sd_shard_args (include/specdec_b200.h)."""
    _fields_ = [("tgt", _vp), ("tgt_bs", _i64), ("tgt_ps", _i64),
                ("drf", _vp), ("drf_bs", _i64), ("drf_ps", _i64),
                ("dtype", _i32),
                ("xs", _vp), ("xs_bs", _i64),
                ("u_acc", _vp), ("u_bs", _i64),
                ("u_res", _vp), ("alive", _vp),
                ("B", _i32), ("k", _i32), ("V", _i32), ("rank", _i32), ("nranks", _i32),
                ("v_start", _i32 * (SHARD_MAX_RANKS + 1)),
                ("temperature", _f32), ("top_p", _f32), ("top_k", _i32),
                ("n_acc", _vp), ("y", _vp),
                ("workspace", _vp), ("workspace_bytes", _sz)]

_lib = None
_lock = threading.Lock()


class SpecdecError(RuntimeError):
    pass


def lib():
    """The loaded library (raises if it was not built)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not LIB_PATH.exists():
                    raise SpecdecError(
                        f"{LIB_PATH.name} is not built; run adaptive-specdec_b200/build.py "
                        "(the verify-round kernels have no CPU fallback)")
                handle = ctypes.CDLL(str(LIB_PATH))
                for name, (args, res) in _SIGNATURES.items():
                    fn = getattr(handle, name, None)
                    if fn is None:
                        continue
                    fn.argtypes = args
                    fn.restype = res
                _lib = handle
    return _lib


def exported_symbols():
    """Names declared in the header that the loaded library exports."""
    h = lib()
    return [n for n in _SIGNATURES if getattr(h, n, None) is not None]


def check(rc, what):
    if rc != 0:
        raise SpecdecError(f"{what} failed: {ERRORS.get(rc, 'error')} (code {rc})")


def require_cuda(*tensors):
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise SpecdecError("specdec_b200 kernels need CUDA tensors (no CPU fallback)")


def ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream_ptr(device=None):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def dtype_code(dt):
    if dt not in SD_DTYPE:
        raise SpecdecError(f"unsupported logits dtype {dt}")
    return SD_DTYPE[dt]


class _Workspaces:
    """Per (device, stream) scratch, grown on demand.

    Each call zeroes the completion counters it uses (the greedy calls use
    none), so a workspace is reusable by any later call on the same stream;
    one per stream keeps calls on different streams from overlapping in the
    same scratch.
    """

    def __init__(self):
        self._ws = {}

    def get(self, nbytes, device):
        key = (device.index, torch.cuda.current_stream(device).cuda_stream)
        cur = self._ws.get(key)
        if cur is None or cur.numel() < nbytes:
            cur = torch.zeros(max(int(nbytes), 1 << 20), dtype=torch.uint8, device=device)
            self._ws[key] = cur
        return cur


workspaces = _Workspaces()
