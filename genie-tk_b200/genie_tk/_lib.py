"""Loader of the C-ABI library ``lib/libgenie_tk_b200.so`` (ctypes).

The library is the only compute path of this package. If it is missing or cannot be
loaded, every op raises ``RuntimeError`` -- there is no fallback.
"""

from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("GENIE_TK_B200_LIB", os.path.join(_HERE, "lib", "libgenie_tk_b200.so"))

_lock = threading.Lock()
_lib = None
_load_error = None

c_i64 = ctypes.c_int64
c_int = ctypes.c_int
c_vp = ctypes.c_void_p
c_size = ctypes.c_size_t

# Return codes of include/genie_tk_b200.h (tests/test_capi_cpu.py checks that these match
# the header).
GTK_OK = 0
GTK_ERR_INVALID_ARG = -1
GTK_ERR_UNSUPPORTED = -2
GTK_ERR_ALIGNMENT = -3
GTK_ERR_WORKSPACE = -4
GTK_ERR_CUDA = -5
GTK_ERR_TMAP = -6
GTK_ERR_DEVICE = -7


class TrimulParams(ctypes.Structure):
    """Mirror of ``gtk_trimul_params`` (include/genie_tk_b200.h)."""

    _fields_ = [(name, c_vp) for name in (
        "ln_in_w", "ln_in_b", "a_p_w", "a_p_b", "a_g_w", "a_g_b", "b_p_w", "b_p_b", "b_g_w", "b_g_b",
        "g_w", "g_b", "z_w", "z_b", "ln_out_w", "ln_out_b")]


class TriattParams(ctypes.Structure):
    """Mirror of ``gtk_triatt_params`` (include/genie_tk_b200.h)."""

    _fields_ = [(name, c_vp) for name in (
        "ln_w", "ln_b", "bias_w", "q_w", "k_w", "v_w", "g_w", "g_b", "o_w", "o_b")]


class TransitionParams(ctypes.Structure):
    """Mirror of ``gtk_transition_params`` (include/genie_tk_b200.h)."""

    _fields_ = [(name, c_vp) for name in ("ln_w", "ln_b", "w1", "b1", "w2", "b2")]


class Dropout(ctypes.Structure):
    """Mirror of ``gtk_dropout`` (include/genie_tk_b200.h)."""

    _fields_ = [("keep_bits", c_vp), ("scale", ctypes.c_float), ("shared_across_rows", c_int)]


# name -> (restype, argtypes)
_SIGNATURES = {
    "gtk_version": (c_int, []),
    "gtk_last_error_string": (ctypes.c_char_p, []),
    "gtk_plane_pitch": (c_i64, [c_i64]),
    "gtk_trimul_packed_bytes": (c_size, [c_int, c_int]),
    "gtk_trimul_pack": (c_int, [ctypes.POINTER(TrimulParams), c_int, c_int, c_vp, c_size, c_vp]),
    "gtk_trimul_workspace_bytes": (c_size, [c_i64, c_i64, c_int, c_int]),
    "gtk_trimul_forward": (c_int, [c_int, c_vp, c_vp, c_vp, c_vp, c_int, c_vp, c_size, c_i64, c_i64, c_int, c_int,
                                   c_vp, c_vp]),
    "gtk_trimul_forward_noalloc": (c_int, [c_int, c_vp, c_vp, c_vp, c_vp, c_int, c_i64, c_i64, c_int, c_int, c_vp,
                                           c_vp]),
    "gtk_trimul_project": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, c_vp, c_vp]),
    "gtk_trimul_project_sharded": (c_int, [c_vp, c_vp, c_vp, ctypes.POINTER(c_vp), ctypes.POINTER(c_vp), c_int,
                                           c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_vp, c_vp]),
    "gtk_trimul_contract": (c_int, [c_int, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64,
                                    ctypes.c_float, c_vp, c_vp]),
    "gtk_trimul_finish": (c_int, [c_vp, c_vp, c_i64, ctypes.c_float, c_vp, c_vp, c_int, c_i64, c_i64, c_i64, c_vp,
                                  c_vp]),
    "gtk_triatt_packed_bytes": (c_size, [c_int, c_int, c_int]),
    "gtk_triatt_pack": (c_int, [ctypes.POINTER(TriattParams), c_int, c_int, c_int, c_vp, c_size, c_vp]),
    "gtk_triatt_workspace_bytes": (c_size, [c_i64, c_i64, c_int, c_int, c_int]),
    "gtk_triatt_forward": (c_int, [c_int, c_vp, c_vp, c_vp, c_vp, c_int, c_vp, c_size, c_i64, c_i64, c_int, c_int,
                                   c_int, ctypes.c_float, c_vp, c_vp]),
    "gtk_triatt_project": (c_int, [c_int, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, c_vp, c_vp]),
    "gtk_triatt_core": (c_int, [c_int, c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, ctypes.c_float, c_vp, c_vp]),
    "gtk_triatt_finish": (c_int, [c_int, c_vp, c_vp, c_vp, c_vp, c_int, c_i64, c_i64, c_i64, c_vp, c_vp]),
    "gtk_triatt_workspace_offsets": (c_int, [c_i64, c_i64, c_i64, ctypes.POINTER(c_i64)]),
    "gtk_copy_2d": (c_int, [c_vp, c_i64, c_vp, c_i64, c_i64, c_i64, c_vp]),
    "gtk_copy_3d": (c_int, [c_vp, c_i64, c_i64, c_vp, c_i64, c_i64, c_i64, c_i64, c_i64, c_vp]),
    "gtk_copy_2d_dma": (c_int, [c_vp, c_i64, c_vp, c_i64, c_i64, c_i64, c_vp]),
    "gtk_pair_transpose_pack": (c_int, [c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, c_vp]),
    "gtk_peer_alloc": (c_int, [c_size, ctypes.POINTER(c_vp), c_vp]),
    "gtk_peer_free": (c_int, [c_vp]),
    "gtk_peer_open": (c_int, [c_vp, ctypes.POINTER(c_vp)]),
    "gtk_peer_close": (c_int, [c_vp]),
    "gtk_push_3d": (c_int, [c_vp, c_int, c_i64, c_i64, c_vp, c_i64, c_i64, c_i64, c_i64, c_vp]),
    "gtk_push_pair_transpose": (c_int, [c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_vp]),
    "gtk_peer_barrier": (c_int, [c_vp, c_int, c_int, ctypes.c_uint32, c_vp, c_vp]),
    "gtk_transition_packed_bytes": (c_size, [c_int, c_int]),
    "gtk_transition_pack": (c_int, [ctypes.POINTER(TransitionParams), c_int, c_int, c_vp, c_size, c_vp]),
    "gtk_transition_workspace_bytes": (c_size, [c_i64, c_i64, c_int, c_int]),
    "gtk_transition_forward": (c_int, [c_vp, c_vp, c_vp, c_vp, c_int, c_vp, c_size, c_i64, c_i64, c_int, c_int, c_vp,
                                       c_vp]),
    "gtk_pair_embed_workspace_bytes": (c_size, [c_i64, c_i64, c_int]),
    "gtk_pair_embed": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_size, c_i64, c_i64, c_i64, c_i64, c_int,
                               c_int, c_vp]),
    "gtk_dropout_keep_bits_philox": (c_int, [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_double, c_i64, c_vp, c_vp]),
    "gtk_dropout_pack_keep_bits": (c_int, [c_vp, c_i64, c_vp, c_vp]),
    "gtk_layernorm": (c_int, [c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, ctypes.c_float, c_vp]),
    "gtk_attn_core_forward": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_int, c_int, ctypes.c_float,
                                      c_vp, c_vp, c_vp]),
    "gtk_attn_core_backward": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, ctypes.c_float, c_i64, c_i64,
                                       c_int, c_int, ctypes.c_float, c_vp, c_vp, c_vp, c_vp, c_vp]),
    "gtk_attn_core_packed_bytes": (c_size, [c_i64, c_i64, c_int, c_int]),
    "gtk_attn_core_bias_bytes": (c_size, [c_i64, c_i64, c_int]),
    "gtk_attn_core_pack": (c_int, [c_vp, c_i64, c_i64, c_int, c_int, ctypes.c_float, c_vp, c_vp]),
    "gtk_attn_core_pack_bias": (c_int, [c_vp, c_i64, c_i64, c_int, c_vp, c_vp]),
    "gtk_trimul_contract_to_peers": (c_int, [c_int, c_vp, c_vp, c_vp, c_int, c_i64, c_i64, c_i64, c_i64, c_i64,
                                             c_i64, c_i64, c_i64, c_i64, c_i64, ctypes.c_float, c_vp, c_vp]),
    "gtk_triatt_finish_to_peers": (c_int, [c_vp, c_vp, c_vp, c_vp, c_int, c_i64, c_i64, c_i64, c_i64, c_int, c_vp,
                                           c_vp]),
    "gtk_mha_forward": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, c_int, c_int,
                                ctypes.c_float, c_vp, c_vp]),
    "gtk_layernorm_linear": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, ctypes.c_float, c_vp]),
    "gtk_linear": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_vp]),
    "gtk_trimul_forward_dropout": (c_int, [c_int, c_vp, c_vp, c_vp, c_vp, c_int, ctypes.POINTER(Dropout), c_vp, c_size,
                                           c_i64, c_i64, c_int, c_int, c_vp, c_vp]),
    "gtk_triatt_forward_dropout": (c_int, [c_int, c_vp, c_vp, c_vp, c_vp, c_int, ctypes.POINTER(Dropout), c_vp, c_size,
                                           c_i64, c_i64, c_int, c_int, c_int, ctypes.c_float, c_vp, c_vp]),
}


def exported_names():
    return list(_SIGNATURES)


def load(required: bool = True):
    """Load (once) and return the ctypes library; raise RuntimeError if ``required`` and absent."""
    global _lib, _load_error
    with _lock:
        if _lib is None and _load_error is None:
            try:
                lib = ctypes.CDLL(LIB_PATH)
                for name, (res, args) in _SIGNATURES.items():
                    fn = getattr(lib, name, None)
                    if fn is None:
                        continue
                    fn.restype = res
                    fn.argtypes = args
                _lib = lib
            except OSError as e:  # pragma: no cover - depends on the build
                _load_error = f"cannot load {LIB_PATH}: {e}"
    if _lib is None and required:
        raise RuntimeError(_load_error or f"cannot load {LIB_PATH}")
    return _lib


def available() -> bool:
    return load(required=False) is not None


def check(rc: int, what: str) -> None:
    if rc != 0:
        msg = load().gtk_last_error_string()
        raise RuntimeError(f"{what} failed ({rc}): {msg.decode() if msg else ''}")
