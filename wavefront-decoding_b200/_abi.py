"""ctypes binding of libwfd_b200.so (include/wfd_b200.h).

The library is the product: every attention / KV-slot operation of this
package goes through these entry points.  Loading fails loudly when the built
library is missing — there is no Python or CPU fallback.
"""
from __future__ import annotations

import ctypes
import pathlib
import threading

_PKG_DIR = pathlib.Path(__file__).resolve().parent
LIB_PATH = _PKG_DIR / "_lib" / "libwfd_b200.so"

WFD_OK = 0
WFD_DTYPE_BF16 = 0
WFD_DTYPE_F32 = 1

# every symbol include/wfd_b200.h declares
EXPORTED = (
    "wfd_abi_version", "wfd_status_string", "wfd_read_error", "wfd_workspace_bytes", "wfd_workspace_init",
    "wfd_wave_attn", "wfd_wave_attn_static", "wfd_wave_attn_kernel", "wfd_attn_varlen", "wfd_attn_segments",
    "wfd_attn_prefill", "wfd_wave_attn_rows",
    "wfd_append",
    "wfd_write_prefill", "wfd_commit_drop", "wfd_commit_window", "wfd_gather_pack",
    "wfd_rmsnorm", "wfd_rope_split", "wfd_silu_mul", "wfd_gather_rows", "wfd_scatter_rows",
    "wfd_items_from_table", "wfd_argmax_rows",
    "wfd_sched_pre_tick", "wfd_sched_route", "wfd_sched_settle", "wfd_sched_params_bytes",
    "wfd_set_batch_invariant", "wfd_get_batch_invariant", "wfd_test_fail_waits",
    "wfd_linear", "wfd_linear_params_bytes", "wfd_rope_split_norm", "wfd_silu_mul_norm",
)

WFD_LINEAR_PLAIN, WFD_LINEAR_RESIDUAL, WFD_LINEAR_SWIGLU, WFD_LINEAR_ROPE = 0, 1, 2, 3


class WfdError(RuntimeError):
    """A libwfd_b200 entry point returned a non-zero status."""

    def __init__(self, what: str, status: int, detail: str):
        super().__init__(f"{what}: status {status} ({detail})")
        self.status = status


class wfd_item(ctypes.Structure):
    _fields_ = [("slot", ctypes.c_int32), ("seq", ctypes.c_int32), ("pos0", ctypes.c_int32),
                ("q_len", ctypes.c_int32), ("q_row0", ctypes.c_int32)]


ABI_VERSION = 6  # include/wfd_b200.h: WFD_ABI_VERSION (declarations and struct layouts below)


class wfd_sched_params(ctypes.Structure):
    """include/wfd_b200.h: wfd_sched_params (field order and types must match)."""
    _fields_ = [(n, ctypes.c_void_p) for n in (
        "alive", "state", "tok", "pos", "step", "n_commit", "done", "committed", "seq_ct", "emu", "emu_ctr",
        "batch_ct", "keys", "c_slot", "lens", "err", "p_tab", "r_tab", "c_tab", "c_out")] + \
        [(n, ctypes.c_int32) for n in (
            "B", "W", "T_total", "T_draft", "max_new", "emu_len", "n_core", "n_kv_slots", "lens_stride",
            "max_seq", "p_cols", "c_cols", "r_cap", "scratch_row", "scratch_seq", "p_slot0", "n_prelude",
            "c_slot0", "n_coda", "depth_slots", "gap_windows")]


class wfd_linear_params(ctypes.Structure):
    """include/wfd_b200.h: wfd_linear_params (field order and types must match)."""
    _fields_ = [(n, ctypes.c_void_p) for n in (
        "x", "w", "out", "q", "k", "v", "cos_tab", "sin_tab", "pos", "err")] + \
        [(n, ctypes.c_int32) for n in ("n_rows", "K", "F", "ldx", "ldo", "mode", "row_norm")] + \
        [("eps", ctypes.c_float)] + \
        [(n, ctypes.c_int32) for n in ("H", "Hkv", "Dh", "rope_style", "pos_stride", "pos_period", "max_pos")]


_P = ctypes.c_void_p
_I = ctypes.c_int32
_F = ctypes.c_float
_S = ctypes.c_size_t

_SIGS = {
    "wfd_abi_version": ([], _I),
    "wfd_sched_params_bytes": ([], _S),
    "wfd_status_string": ([_I], ctypes.c_char_p),
    "wfd_read_error": ([_P, _P, _P], _I),
    "wfd_workspace_bytes": ([_I, _I, _I], _S),
    "wfd_workspace_init": ([_P, _S, _P], _I),
    # q k_new v_new kc vc out lens items n max_q slot_off n_rows n_slots n_seqs max_seq Hq Hkv Dh dtype scale ws ws_bytes err stream
    "wfd_wave_attn": ([_P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I, _I, _I, _I, _F, _P, _S, _P, _P], _I),
    "wfd_wave_attn_kernel": ([_I, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I, _I, _I, _I, _F, _P, _S,
                              _P, _P], _I),
    # which q k_new v_new kc vc out lens items n max_q row_pos rp_stride slot_off n_rows n_slots n_seqs max_seq Hq Hkv
    # Dh dtype scale ws ws_bytes err stream
    "wfd_wave_attn_rows": ([_I, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _P, _I, _I, _I, _I, _I, _I, _I, _I, _I, _I, _F,
                            _P, _S, _P, _P], _I),
    # as wfd_wave_attn without (ws, ws_bytes)
    "wfd_wave_attn_static": ([_P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I, _I, _I, _I, _F, _P, _P], _I),
    # q k v out cu_q cu_k n max_q total_q total_k Hq Hkv Dh dtype causal scale ws ws_bytes err stream
    "wfd_attn_varlen": ([_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I, _I, _F, _P, _S, _P, _P], _I),
    # q k v out q_row0 q_len k_row0 k_len n max_q total_q total_k Hq Hkv Dh dtype causal scale ws ws_bytes err stream
    "wfd_attn_segments": ([_P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I, _I, _F, _P, _S, _P, _P], _I),
    # q k v out n_seqs q_len k_len Hq Hkv Dh dtype causal scale err stream
    "wfd_attn_prefill": ([_P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I, _F, _P, _P], _I),
    # k_new v_new kc vc lens slots seqs positions n slot_off n_slots n_seqs max_seq Hkv Dh dtype err stream
    "wfd_append": ([_P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I, _P, _P], _I),
    # k v kc vc lens slot L n_slots n_seqs max_seq Hkv Dh dtype stream
    "wfd_write_prefill": ([_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I, _P], _I),
    "wfd_commit_drop": ([_P, _P, _I, _I, _P], _I),
    # kc vc lens items n accept_len accept_mask acc_rows acc_count n_rows slot_off n_slots n_seqs max_seq Hkv Dh dtype
    # err stream
    "wfd_commit_window": ([_P, _P, _P, _P, _I, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I, _P, _P], _I),
    # kc vc kp vp slots seqs cu_k n n_slots n_seqs max_seq Hkv Dh dtype err stream
    "wfd_gather_pack": ([_P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _P, _P], _I),
    # x w y n d eps dtype stream
    "wfd_rmsnorm": ([_P, _P, _P, _I, _I, _F, _I, _P], _I),
    # qkv cos sin pos pos_stride pos_period max_pos q k v n H Hkv Dh style dtype err stream
    "wfd_rope_split": ([_P, _P, _P, _P, _I, _I, _I, _P, _P, _P, _I, _I, _I, _I, _I, _I, _P, _P], _I),
    # gu out n dff dtype stream
    "wfd_silu_mul": ([_P, _P, _I, _I, _I, _P], _I),
    # qkv x ldx d eps cos sin pos pos_stride pos_period max_pos q k v n H Hkv Dh style dtype err stream
    "wfd_rope_split_norm": ([_P, _P, _I, _I, _F, _P, _P, _P, _I, _I, _I, _P, _P, _P, _I, _I, _I, _I, _I, _I, _P, _P],
                            _I),
    # gu x ldx d eps out n dff dtype stream
    "wfd_silu_mul_norm": ([_P, _P, _I, _I, _F, _P, _I, _I, _I, _P], _I),
    # a b idx stride out n d n_src dtype err stream
    "wfd_gather_rows": ([_P, _P, _P, _I, _P, _I, _I, _I, _I, _P, _P], _I),
    # src idx stride dst zero n d n_dst dtype err stream
    "wfd_scatter_rows": ([_P, _P, _I, _P, _P, _I, _I, _I, _I, _P, _P], _I),
    # tab cols c_slot c_seq c_pos c_qlen items n stream
    "wfd_items_from_table": ([_P, _I, _I, _I, _I, _I, _P, _I, _P], _I),
    # x out n V dtype stream
    "wfd_argmax_rows": ([_P, _P, _I, _I, _I, _P], _I),
    "wfd_set_batch_invariant": ([_I], _I),
    "wfd_get_batch_invariant": ([], _I),
    "wfd_test_fail_waits": ([_I], _I),
    # const wfd_linear_params*, stream
    "wfd_linear": ([_P, _P], _I),
    "wfd_linear_params_bytes": ([], _S),
    # const wfd_sched_params*, stream
    "wfd_sched_pre_tick": ([_P, _P], _I),
    "wfd_sched_route": ([_P, _P], _I),
    "wfd_sched_settle": ([_P, _P], _I),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Load libwfd_b200.so once and attach the C signatures."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise ImportError(
                f"libwfd_b200.so not found at {LIB_PATH}; build it with "
                "`python wavefront-decoding_b200/build.py` (nvcc, sm_100a)")
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (args, res) in _SIGS.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = res
        if lib.wfd_abi_version() != ABI_VERSION:
            raise ImportError(f"{LIB_PATH} has ABI version {lib.wfd_abi_version()}, these bindings expect "
                              f"{ABI_VERSION}: rebuild it (`python wavefront-decoding_b200/build.py`)")
        _lib = lib
    return _lib


def status_string(status: int) -> str:
    return load().wfd_status_string(status).decode()


def check(status: int, what: str) -> None:
    if status != WFD_OK:
        raise WfdError(what, status, status_string(status))
