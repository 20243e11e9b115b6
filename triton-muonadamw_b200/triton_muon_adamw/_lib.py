"""ctypes binding of the C ABI declared in ``include/muon_adamw_b200.h``.

The shared library ``libmuonadamw_b200.so`` is built in-tree next to this file
(``python -m triton_muon_adamw._build``).  Loading fails loudly if it is
missing: the optimizer has no other implementation.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

LIB_NAME = "libmuonadamw_b200.so"
ABI_VERSION = 4  # mad_abi_version() of the library these structures describe
DTYPE_F32, DTYPE_BF16, DTYPE_F32_MASTER = 0, 1, 2  # MAD_DTYPE_*
ERR_DEVICE = 5            # MAD_ERR_DEVICE: a kernel reported an error in its status word
# Status bits of the Muon kernels (a barrier wait that gave up, by role).
DEV_ERR_TIMEOUT_PRODUCER, DEV_ERR_TIMEOUT_MMA, DEV_ERR_TIMEOUT_EPILOGUE, DEV_ERR_TIMEOUT_DRAIN = 1, 2, 4, 8
LIB_PATH = Path(__file__).resolve().parent / LIB_NAME

c_int32 = ctypes.c_int32
c_int64 = ctypes.c_int64
c_float = ctypes.c_float
c_void_p = ctypes.c_void_p


class AdamWTensor(ctypes.Structure):
    _fields_ = [("param", c_void_p), ("grad", c_void_p), ("exp_avg", c_void_p), ("exp_avg_sq", c_void_p),
                ("numel", c_int64), ("dtype", c_int32), ("pad", c_int32), ("shadow", c_void_p)]


class MuonMatrix(ctypes.Structure):
    _fields_ = [("param", c_void_p), ("grad", c_void_p), ("momentum", c_void_p), ("rows", c_int64),
                ("cols", c_int64), ("lr_scale", ctypes.c_double), ("dtype", c_int32), ("pad", c_int32),
                ("shadow", c_void_p)]


class MuonPlanInfo(ctypes.Structure):
    _fields_ = [("n_mats", c_int32), ("num_sms", c_int32), ("table_bytes", c_int64), ("work_bytes", c_int64),
                ("prep_tiles", c_int64), ("gram_tiles", c_int64), ("poly_tiles", c_int64),
                ("update_tiles", c_int64), ("off_mats", c_int64), ("off_tmaps", c_int64),
                ("off_gram_tiles", c_int64), ("off_poly_tiles", c_int64), ("off_update_tiles", c_int64),
                ("off_prep_map", c_int64), ("off_partials", c_int64)]


class MuonBuffers(ctypes.Structure):
    _fields_ = [("x", c_void_p * 2), ("gram", c_void_p), ("poly", c_void_p), ("m", c_int64), ("n", c_int64),
                ("ld_x", c_int64), ("ld_mm", c_int64), ("transposed", c_int32)]


MAX_RANKS = 8            # MAD_MAX_RANKS
IPC_HANDLE_BYTES = 64    # MAD_IPC_HANDLE_BYTES


class GradReduce(ctypes.Structure):
    _fields_ = [("n_ranks", c_int32), ("scale", c_float), ("delta", c_int64 * MAX_RANKS)]


class PeerSet(ctypes.Structure):
    _fields_ = [("n_peers", c_int32), ("pad", c_int32), ("delta", c_int64 * MAX_RANKS)]


# name -> (restype, argtypes); every entry point declared in include/muon_adamw_b200.h
SIGNATURES = {
    "mad_last_error": (ctypes.c_char_p, []),
    "mad_abi_version": (c_int32, []),
    "mad_adamw_step": (ctypes.c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_float, c_float, c_float,
                                      c_float, c_float, c_float, c_float, c_void_p]),
    "mad_adamw_table_bytes": (ctypes.c_int, [ctypes.POINTER(AdamWTensor), c_int32, ctypes.POINTER(c_int64)]),
    "mad_adamw_plan": (ctypes.c_int, [ctypes.POINTER(AdamWTensor), c_int32, c_void_p, c_int64,
                                      ctypes.POINTER(c_int64), c_void_p]),
    "mad_adamw_step_multi": (ctypes.c_int, [c_void_p, c_int64, c_float, c_float, c_float, c_float, c_float, c_float,
                                            c_float, c_void_p]),
    "mad_adamw_step_multi_reduce": (ctypes.c_int, [c_void_p, c_int64, c_float, c_float, c_float, c_float, c_float,
                                                   c_float, c_float, ctypes.POINTER(GradReduce), c_void_p]),
    "mad_muon_plan_size": (ctypes.c_int, [ctypes.POINTER(MuonMatrix), c_int32, ctypes.POINTER(MuonPlanInfo)]),
    "mad_muon_plan": (ctypes.c_int, [ctypes.POINTER(MuonMatrix), c_int32, c_void_p, c_void_p,
                                     ctypes.POINTER(MuonPlanInfo), ctypes.POINTER(MuonBuffers), c_void_p]),
    "mad_muon_prep": (ctypes.c_int, [ctypes.POINTER(MuonPlanInfo), c_void_p, ctypes.c_double, c_int32, c_float,
                                     c_void_p]),
    "mad_muon_prep_reduce": (ctypes.c_int, [ctypes.POINTER(MuonPlanInfo), c_void_p, ctypes.c_double, c_int32,
                                            c_float, ctypes.POINTER(GradReduce), c_void_p]),
    "mad_ns_gram": (ctypes.c_int, [ctypes.POINTER(MuonPlanInfo), c_void_p, c_int32, c_void_p]),
    "mad_ns_poly": (ctypes.c_int, [ctypes.POINTER(MuonPlanInfo), c_void_p, c_int32, c_float, c_float, c_void_p]),
    "mad_ns_update": (ctypes.c_int, [ctypes.POINTER(MuonPlanInfo), c_void_p, c_int32, c_int32, c_float,
                                     ctypes.c_double, ctypes.c_double, c_void_p]),
    "mad_muon_step_multi": (ctypes.c_int, [ctypes.POINTER(MuonPlanInfo), c_void_p, ctypes.c_double, c_int32, c_float,
                                           c_float, c_float, c_int32, c_float, ctypes.c_double, ctypes.c_double,
                                           c_void_p]),
    "mad_muon_step_multi_reduce": (ctypes.c_int, [ctypes.POINTER(MuonPlanInfo), c_void_p, ctypes.c_double, c_int32,
                                                  c_float, c_float, c_float, c_int32, c_float, ctypes.c_double,
                                                  ctypes.c_double, ctypes.POINTER(GradReduce), c_void_p]),
    "mad_muon_step_noalloc": (ctypes.c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, ctypes.c_double,
                                             ctypes.c_double, c_int32, c_float, c_float, c_float, c_int32, c_float,
                                             ctypes.c_double, ctypes.c_double, c_void_p]),
    "mad_muon_read_status": (ctypes.c_int, [ctypes.POINTER(MuonPlanInfo), c_void_p, ctypes.POINTER(ctypes.c_uint32),
                                            c_int32, c_void_p]),
    "mad_ipc_alloc": (ctypes.c_int, [c_int64, ctypes.POINTER(c_void_p), c_void_p]),
    "mad_ipc_free": (ctypes.c_int, [c_void_p]),
    "mad_ipc_open": (ctypes.c_int, [c_void_p, ctypes.POINTER(c_void_p)]),
    "mad_ipc_close": (ctypes.c_int, [c_void_p]),
    "mad_copy_async": (ctypes.c_int, [c_void_p, c_void_p, c_int64, c_void_p]),
    "mad_peer_push": (ctypes.c_int, [c_void_p, c_int64, ctypes.POINTER(PeerSet), c_void_p]),
    "mad_debug_expire_next_waits": (ctypes.c_int, [c_int32]),
    "mad_set_gemm_sm_reserve": (ctypes.c_int, [c_int32]),
    "mad_adamw_set_grads": (ctypes.c_int, [c_void_p, c_int64, ctypes.POINTER(c_void_p), c_int32, c_void_p]),
    "mad_muon_set_grads": (ctypes.c_int, [ctypes.POINTER(MuonPlanInfo), c_void_p, ctypes.POINTER(c_void_p),
                                          c_void_p]),
}

_lib = None


class MuonAdamWLibraryError(RuntimeError):
    """A C-ABI call returned a non-zero status."""


def load():
    """Load (once) and return the CUDA library, with argument types declared."""
    global _lib
    if _lib is not None:
        return _lib
    path = Path(os.environ.get("MUON_ADAMW_B200_LIB", str(LIB_PATH)))
    if not path.exists():
        raise ImportError(f"{path} is missing: build the CUDA library first "
                          "(python -m triton_muon_adamw._build); there is no fallback implementation")
    lib = ctypes.CDLL(str(path))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    version = lib.mad_abi_version()
    if version != ABI_VERSION:
        raise ImportError(f"{path} has ABI version {version}, these bindings need {ABI_VERSION}: rebuild it "
                          "(python -m triton_muon_adamw._build)")
    _lib = lib
    return lib


def check(rc: int, what: str = "") -> None:
    if rc != 0:
        msg = load().mad_last_error().decode(errors="replace")
        raise MuonAdamWLibraryError(f"{what or 'muon_adamw_b200'} failed with status {rc}: {msg}")


def stream_handle(stream=None) -> int:
    """Raw cudaStream_t of the given (or current) torch stream."""
    import torch  # noqa: PLC0415
    s = stream if stream is not None else torch.cuda.current_stream()
    return int(s.cuda_stream)
