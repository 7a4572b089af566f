"""ctypes binding of libflux_b200.so (the C-ABI declared in include/flux_b200.h).

The library is loaded from ``selas_b200/lib/libflux_b200.so`` (built in-tree by
``python -m selas_b200.build``). There is no fallback: if the library is missing or does not load,
every entry point raises ``FluxB200Error``.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libflux_b200.so"

FB_F32, FB_F16, FB_BF16 = 0, 1, 2
FB_PROBE_WORK_DOUBLES = 4096
FB_VAE_ROUND_OUT, FB_VAE_OUT_NCHW_CLAMP = 1, 2
FB_EPI_STORE_BF16, FB_EPI_STORE_F32, FB_EPI_GELU, FB_EPI_GATED_RESIDUAL, FB_EPI_QKV = range(5)
DEVICE_CODES = {0: "ok", 1: "timeout waiting for TMA", 2: "timeout waiting for tensor-core work",
                3: "timeout waiting for epilogue/softmax warps", 4: "bad shape seen on the device",
                5: "timeout waiting for another rank at a peer barrier"}

# Every symbol include/flux_b200.h declares, with its ctypes signature.
_P, _I32, _I64, _F = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_float
SIGNATURES = {
    "fb_init": ([], _I32),
    "fb_last_error": ([], ctypes.c_char_p),
    "fb_device_status": ([ctypes.POINTER(_I32), _I32], _I32),
    "fb_version": ([], ctypes.c_char_p),
    "fb_selftest_wait_timeout": ([_I32, _P], _I32),
    "fb_attention_sp": ([_P, _P, _P, _P, _I64, _I32, _I32, _I32, _I32, _I32, _F, _P], _I32),
    "fb_ipc_export": ([_P, _P, ctypes.POINTER(_I64)], _I32),
    "fb_ipc_open": ([_P, _I64, ctypes.POINTER(_P), ctypes.POINTER(_P)], _I32),
    "fb_ipc_close": ([_P], _I32),
    "fb_peer_barrier": ([_P, _I32, _I32, _I32, _I32, _P], _I32),
    "fb_nf4_encode": ([_P, _I32, _I64, _I32, _P, _P, _P, _P], _I32),
    "fb_int8_row_encode": ([_P, _I32, _I64, _I64, _P, _P, _P], _I32),
    "fb_probe_distance": ([_P, _P, _P, _P, _I64, _P, _P], _I32),
    "fb_residual_predict": ([_P, _P, _P, _I32, _F, _P, _I64, _P], _I32),
    "fb_residual_diff": ([_P, _P, _P, _I32, _I64, _P], _I32),
    "fb_vae_conv": ([_P, _I64, _I32, _I32, _I32, _I32, _P, _I64, _I32, _I32, _P, _P, _I64, _P, _I64, _I32, _P], _I32),
    "fb_vae_group_norm": ([_P, _I64, _I32, _I64, _I32, _P, _P, _F, _I32, _I32, _P, _I64, _P, _P], _I32),
    "fb_vae_group_norm_work_doubles": ([_I32], _I64),
    "fb_vae_norm_out_conv": ([_P, _I32, _I32, _I32, _I32, _P, _P, _F, _P, _P, _I32, _P, _P, _P], _I32),
    "fb_vae_upsample2": ([_P, _I32, _I32, _I32, _I32, _I32, _P, _P], _I32),
    "fb_vae_softmax_rows": ([_P, _I64, _I32, _I64, _F, _I32, _P], _I32),
    "fb_vae_transpose": ([_P, _I32, _I32, _I64, _P, _I64, _P], _I32),
    "fb_vae_latent_prep": ([_P, _I32, _I32, _I32, _I32, _I32, _F, _F, _P, _P], _I32),
    "fb_nf4_dequant": ([_P, _P, _P, _I64, _I32, _P, _I32, _P], _I32),
    "fb_ln_mod": ([_P, _I64, _I32, _I32, _P, _P, _I64, _P, _P], _I32),
    "fb_ln_mod_grouped": ([_P, _I32, _P], _I32),
    "fb_linear_grouped": ([_P, _I32, _I32, _P], _I32),
    "fb_linear_nf4": ([_P, _I32, _P, _I64, _P], _I32),
    "fb_linear_nf4_static": ([_P, _I32, _P], _I32),
    "fb_linear_nf4_static_status": ([ctypes.POINTER(_I32), _I32], _I32),
    "fb_selftest_static_wait_timeout": ([_I32, _P], _I32),
    "fb_attention": ([_P, _P, _P, _P, _I64, _I32, _I32, _I32, _I32, _F, _P], _I32),
    "fb_attention_split": ([_P, _P, _P, _P, _I64, _P, _I64, _I32, _I32, _I32, _I32, _I32, _F, _P], _I32),
    "fb_gated_add": ([_P, _P, _P, _P, _I64, _I32, _I32, _I64, _I32, _P], _I32),
    "fb_gelu_tanh": ([_P, _P, _I64, _P], _I32),
    "fb_qk_norm_rope": ([_P, _I64, _I32, _I32, _I32, _I32, _P, _P, _P, _P, _P, _P, _P, _I32, _I32, _P], _I32),
}


class FluxB200Error(RuntimeError):
    """A libflux_b200 call failed (bad arguments, CUDA error, or a device-side error)."""


class FbLnModProblem(ctypes.Structure):
    """``fb_ln_mod_problem`` of include/flux_b200.h, field for field."""

    _fields_ = [("x", _P), ("rows", _I64), ("dim", _I32), ("rows_per_batch", _I32), ("shift", _P), ("scale", _P),
                ("mod_batch_stride", _I64), ("out", _P)]


class FbLinear(ctypes.Structure):
    """``fb_linear`` of include/flux_b200.h, field for field."""

    _fields_ = [
        ("a", _P), ("lda", _I64),
        ("w", _P), ("ldw", _I64),
        ("w_nf4", _P), ("absmax", _P), ("code16", _P), ("blocksize", _I32),
        ("bias", _P),
        ("m", _I32), ("n", _I32), ("k", _I32),
        ("rows_per_batch", _I32),
        ("out", _P), ("ld_out", _I64),
        ("resid", _P), ("ld_resid", _I64),
        ("gate", _P), ("gate_batch_stride", _I64),
        ("guard", _I32),
        ("q_scale", _P), ("k_scale", _P), ("rope_cos", _P), ("rope_sin", _P),
        ("q", _P), ("k_out", _P), ("v", _P),
        ("heads", _I32), ("head_dim", _I32), ("seq_total", _I32), ("seq_offset", _I32),
        ("qkv_cols", _I32),
        ("gelu_col0", _I32),
        ("w_i8", _P), ("w_scale", _P),
        ("w_f8", _P), ("w_f8_e5m2", _I32),
        ("sp_qkv_dst", _P * 8), ("sp_world", _I32), ("sp_rank", _I32),
    ]


_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def load(path: Path | None = None) -> ctypes.CDLL:
    """Load the library and declare every exported signature (no CUDA call is made)."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = Path(path or LIB_PATH)
        if not p.exists():
            raise FluxB200Error(f"{p} is missing: build it with `python -m selas_b200.build` (no CPU fallback exists)")
        lib = ctypes.CDLL(str(p))
        for name, (args, res) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes, fn.restype = args, res
        if path is None:
            _lib = lib
        return lib


_init_done = False


def lib() -> ctypes.CDLL:
    """The loaded library, initialised for CUDA (fb_init) on first use."""
    global _init_done
    L = load()
    if not _init_done:
        check(L.fb_init(), "fb_init")
        _init_done = True
    return L


def check(rc: int, what: str) -> None:
    if rc != 0:
        msg = load().fb_last_error().decode(errors="replace")
        raise FluxB200Error(f"{what} failed (code {rc}): {msg}")


def device_status(clear: bool = True) -> int:
    """Synchronously read (and clear) the current device's status word; 0 = no device-side error."""
    code = _I32(0)
    check(lib().fb_device_status(ctypes.byref(code), int(clear)), "fb_device_status")
    return int(code.value)


def static_status(clear: bool = True) -> int:
    """Read (and clear) the status word of fb_linear_nf4_static's fixed array without allocating
    anything; 0 = none of its kernels gave up on a wait. Waits for all work on the current device."""
    code = _I32(0)
    L = load()
    check(L.fb_linear_nf4_static_status(ctypes.byref(code), int(clear)), "fb_linear_nf4_static_status")
    return int(code.value)


def raise_on_device_error() -> None:
    """Raise FluxB200Error if a kernel recorded a device-side error: in the library's status word, or in
    the fixed array's word of fb_linear_nf4_static (read only when that entry point has been used)."""
    code = device_status(clear=True)
    if not code and static_used:
        code = static_status(clear=True)
    if code:
        raise FluxB200Error(f"device-side error {code}: {DEVICE_CODES.get(code, 'unknown')}")


static_used = False  # set by ops.run_linear_nf4_static
