"""ctypes binding of libsrs_b200.so (C ABI: include/srs_b200.h).

Everything the package launches goes through ``launcher()``, an object with
one method per C entry point.  There is no fallback: if the library is absent
or the device is not an sm_100a GPU, calls raise.  Tests on machines without a
GPU install a stand-in with ``set_launcher``.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import numpy as np

LIBRARY_PATH = Path(__file__).resolve().parent.parent / "_native" / "libsrs_b200.so"
HOST_PATH = LIBRARY_PATH.parent / "_srs_host.so"

SRS_OK = 0
SRS_ERR_INVALID_ARGUMENT = -1
SRS_ERR_UNSUPPORTED_DEVICE = -2
SRS_ERR_CUDA = -3

ROW_PARAM_BF16 = 0x1
ROW_GRAD_BF16 = 0x2
ROW_VECTOR_OK = 0x4
ROW_CLASS_SHIFT = 8
MAX_STEP_CLASSES = 32
KIND_MIXED = 0xFFFFFFFF
KEY_DERIVE = 0
KEY_GIVEN = 1

# Row table entry (struct srs_row): 64 bytes, 8-byte aligned fields.
ROW_DTYPE = np.dtype([
    ("param", "<u8"), ("grad", "<u8"), ("state", "<u8", (2,)), ("numel", "<i8"),
    ("tile_begin", "<i8"), ("param_index", "<u4"), ("offset", "<u4"), ("flags", "<u4"),
    ("reserved", "<u4"),
])
assert ROW_DTYPE.itemsize == 64


class SrsRow(ctypes.Structure):
    _fields_ = [("param", ctypes.c_uint64), ("grad", ctypes.c_uint64),
                ("state", ctypes.c_uint64 * 2), ("numel", ctypes.c_int64),
                ("tile_begin", ctypes.c_int64), ("param_index", ctypes.c_uint32),
                ("offset", ctypes.c_uint32), ("flags", ctypes.c_uint32),
                ("reserved", ctypes.c_uint32)]


class SrsRng(ctypes.Structure):
    _fields_ = [("seed_lo", ctypes.c_uint32), ("seed_hi", ctypes.c_uint32),
                ("step_lo", ctypes.c_uint32), ("step_hi", ctypes.c_uint32),
                ("key_mode", ctypes.c_int32)]


class SrsAdamWHparams(ctypes.Structure):
    _fields_ = [("beta1", ctypes.c_float), ("beta2", ctypes.c_float),
                ("one_minus_beta1", ctypes.c_float), ("one_minus_beta2", ctypes.c_float),
                ("eps", ctypes.c_float), ("decay", ctypes.c_float),
                ("n_step_classes", ctypes.c_int32),
                ("neg_step_size", ctypes.c_float * MAX_STEP_CLASSES),
                ("bias2_sqrt", ctypes.c_float * MAX_STEP_CLASSES)]


class SrsSgdmHparams(ctypes.Structure):
    _fields_ = [("momentum", ctypes.c_float), ("neg_lr", ctypes.c_float)]


MAX_PEERS = 7
IPC_HANDLE_BYTES = 64


PEERS_STORE, PEERS_MULTICAST = 0, 1


class SrsPeers(ctypes.Structure):
    _fields_ = [("n_peers", ctypes.c_int32), ("mode", ctypes.c_int32),
                ("delta_f32", ctypes.c_int64 * MAX_PEERS),
                ("delta_bf16", ctypes.c_int64 * MAX_PEERS),
                ("mc_delta_f32", ctypes.c_int64), ("mc_delta_bf16", ctypes.c_int64)]


_P = ctypes.c_void_p
_SIGNATURES = {
    "srs_abi_version": ([], ctypes.c_int),
    "srs_tile_elems": ([], ctypes.c_int64),
    "srs_last_error": ([], ctypes.c_char_p),
    "srs_check_device": ([], ctypes.c_int),
    "srs_cast": ([_P, _P, ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_uint32,
                  ctypes.c_uint32, ctypes.c_int, _P], ctypes.c_int),
    "srs_adamw_multi": ([_P, ctypes.c_int64, ctypes.c_int64, ctypes.c_int, ctypes.c_int,
                         ctypes.c_int, ctypes.c_int, ctypes.POINTER(SrsAdamWHparams),
                         ctypes.POINTER(SrsRng), ctypes.c_uint32, ctypes.c_int, _P],
                        ctypes.c_int),
    "srs_sgdm_multi": ([_P, ctypes.c_int64, ctypes.c_int64, ctypes.c_int, ctypes.c_int,
                        ctypes.POINTER(SrsSgdmHparams), ctypes.POINTER(SrsRng), ctypes.c_uint32,
                        ctypes.c_int, _P], ctypes.c_int),
    "srs_adamw_single": ([ctypes.POINTER(SrsRow), ctypes.c_int, ctypes.c_int, ctypes.c_int,
                          ctypes.c_int, ctypes.POINTER(SrsAdamWHparams), ctypes.c_int, _P],
                         ctypes.c_int),
    "srs_sgdm_single": ([ctypes.POINTER(SrsRow), ctypes.c_int, ctypes.c_int,
                         ctypes.POINTER(SrsSgdmHparams), ctypes.c_int, _P], ctypes.c_int),
    "srs_derive_keys": ([_P, _P, ctypes.c_int64, ctypes.POINTER(SrsRng), _P], ctypes.c_int),
    "srs_adamw_multi_noalloc": ([_P, ctypes.c_int64, ctypes.c_int64, ctypes.c_int, ctypes.c_int,
                                 ctypes.c_int, ctypes.c_int, ctypes.POINTER(SrsAdamWHparams),
                                 ctypes.POINTER(SrsRng), ctypes.c_int, _P], ctypes.c_int),
    "srs_adamw_multi_gather": ([_P, ctypes.c_int64, ctypes.c_int64, ctypes.c_int, ctypes.c_int,
                                ctypes.c_int, ctypes.c_int, ctypes.POINTER(SrsAdamWHparams),
                                ctypes.POINTER(SrsRng), ctypes.c_uint32,
                                ctypes.POINTER(SrsPeers), ctypes.c_int, _P], ctypes.c_int),
    "srs_sgdm_multi_gather": ([_P, ctypes.c_int64, ctypes.c_int64, ctypes.c_int, ctypes.c_int,
                               ctypes.POINTER(SrsSgdmHparams), ctypes.POINTER(SrsRng),
                               ctypes.c_uint32, ctypes.POINTER(SrsPeers), ctypes.c_int, _P],
                              ctypes.c_int),
    "srs_adamw_multi_range": ([_P, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                               ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                               ctypes.c_int, ctypes.POINTER(SrsAdamWHparams),
                               ctypes.POINTER(SrsRng), ctypes.c_uint32, ctypes.POINTER(SrsPeers),
                               ctypes.c_int, _P],
                              ctypes.c_int),
    "srs_sgdm_multi_range": ([_P, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                              ctypes.c_int, ctypes.c_int, ctypes.POINTER(SrsSgdmHparams),
                              ctypes.POINTER(SrsRng), ctypes.c_uint32, ctypes.POINTER(SrsPeers),
                              ctypes.c_int, _P],
                             ctypes.c_int),
    "srs_copy_async": ([_P, _P, ctypes.c_uint64, _P], ctypes.c_int),
    "srs_ipc_export": ([_P, _P, ctypes.POINTER(ctypes.c_uint64)], ctypes.c_int),
    "srs_ipc_import": ([_P, ctypes.POINTER(ctypes.c_void_p)], ctypes.c_int),
    "srs_ipc_close": ([_P], ctypes.c_int),
}
NOALLOC_MAX_ROWS = 4096
ABI_VERSION = 6

_lock = threading.Lock()
_library = None


def load_library() -> ctypes.CDLL:
    """Load libsrs_b200.so (raises if it has not been built)."""
    global _library
    with _lock:
        if _library is None:
            if not LIBRARY_PATH.exists():
                raise RuntimeError(
                    f"{LIBRARY_PATH} is missing: build the sm_100a kernels with "
                    "`python stochastic-rounding-pytorch_b200/build_native.py`"
                )
            lib = ctypes.CDLL(str(LIBRARY_PATH))
            for name, (argtypes, restype) in _SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes, fn.restype = argtypes, restype
            if lib.srs_abi_version() != ABI_VERSION:
                raise RuntimeError("libsrs_b200.so ABI version mismatch; rebuild it")
            _library = lib
    return _library


_host = None


def host_module():
    """The _srs_host helper module (raises if it has not been built)."""
    global _host
    if _host is None:
        import importlib.machinery
        import importlib.util

        if not HOST_PATH.exists():
            raise RuntimeError(f"{HOST_PATH} is missing: build it with "
                               "`python stochastic-rounding-pytorch_b200/build_native.py`")
        loader = importlib.machinery.ExtensionFileLoader("_srs_host", str(HOST_PATH))
        spec = importlib.util.spec_from_file_location("_srs_host", str(HOST_PATH), loader=loader)
        module = importlib.util.module_from_spec(spec)
        loader.exec_module(module)
        _host = module
    return _host


def _check(rc: int) -> None:
    if rc == SRS_OK:
        return
    message = load_library().srs_last_error().decode(errors="replace")
    if rc == SRS_ERR_INVALID_ARGUMENT:
        raise ValueError(message)
    raise RuntimeError(message)


class NativeLauncher:
    """Calls into libsrs_b200.so; every method enqueues on ``stream`` (a cudaStream_t)."""

    def __init__(self):
        self._devices_ok: set = set()

    def check_device(self, device, what: str = "fused state updates") -> None:
        """ValueError unless ``device`` is a CUDA device the kernels run on."""
        import torch

        if device.type != "cuda":
            raise ValueError(f"{what} require CUDA tensors")
        index = device.index if device.index is not None else torch.cuda.current_device()
        if index in self._devices_ok:
            return
        major, minor = torch.cuda.get_device_capability(index)
        if (major, minor) != (10, 0):
            raise ValueError(
                f"the sr_states kernels are built for sm_100a (B200, compute capability 10.0); "
                f"cuda:{index} is sm_{major}{minor}"
            )
        load_library()
        self._devices_ok.add(index)

    def tile_elems(self) -> int:
        return int(load_library().srs_tile_elems())

    def cast(self, x_ptr, y_ptr, n, fmt, rule, seed, offset, stream, grid_ctas=0):
        _check(load_library().srs_cast(x_ptr, y_ptr, n, fmt, rule, seed, offset, grid_ctas,
                                       stream))

    def adamw_multi(self, table, n_rows, n_tiles, m_fmt, m_rule, v_fmt, v_rule, hp, rng, stream,
                    grid_ctas=0, peers=None, tiles=None):
        lib = load_library()
        if tiles is not None:
            _check(lib.srs_adamw_multi_range(table.device_ptr, n_rows, n_tiles, tiles[0],
                                             tiles[1], m_fmt, m_rule, v_fmt, v_rule,
                                             ctypes.byref(hp), ctypes.byref(rng),
                                             table.uniform_kind,
                                             None if peers is None else ctypes.byref(peers),
                                             grid_ctas, stream))
        elif peers is None:
            _check(lib.srs_adamw_multi(table.device_ptr, n_rows, n_tiles, m_fmt, m_rule, v_fmt,
                                       v_rule, ctypes.byref(hp), ctypes.byref(rng),
                                       table.uniform_kind, grid_ctas, stream))
        else:
            _check(lib.srs_adamw_multi_gather(table.device_ptr, n_rows, n_tiles, m_fmt, m_rule,
                                              v_fmt, v_rule, ctypes.byref(hp), ctypes.byref(rng),
                                              table.uniform_kind, ctypes.byref(peers), grid_ctas,
                                              stream))

    def sgdm_multi(self, table, n_rows, n_tiles, u_fmt, u_rule, hp, rng, stream, grid_ctas=0,
                   peers=None, tiles=None):
        lib = load_library()
        if tiles is not None:
            _check(lib.srs_sgdm_multi_range(table.device_ptr, n_rows, n_tiles, tiles[0], tiles[1],
                                            u_fmt, u_rule, ctypes.byref(hp), ctypes.byref(rng),
                                            table.uniform_kind,
                                            None if peers is None else ctypes.byref(peers),
                                            grid_ctas, stream))
        elif peers is None:
            _check(lib.srs_sgdm_multi(table.device_ptr, n_rows, n_tiles, u_fmt, u_rule,
                                      ctypes.byref(hp), ctypes.byref(rng), table.uniform_kind,
                                      grid_ctas, stream))
        else:
            _check(lib.srs_sgdm_multi_gather(table.device_ptr, n_rows, n_tiles, u_fmt, u_rule,
                                             ctypes.byref(hp), ctypes.byref(rng),
                                             table.uniform_kind, ctypes.byref(peers), grid_ctas,
                                             stream))

    def copy_async(self, dst, src, nbytes, stream):
        """Device-to-device copy on ``stream`` (peer memory included)."""
        _check(load_library().srs_copy_async(dst, src, nbytes, stream))

    def ipc_export(self, ptr):
        """(handle bytes, offset of ptr in its allocation) for mapping in a peer process."""
        handle = (ctypes.c_char * IPC_HANDLE_BYTES)()
        offset = ctypes.c_uint64()
        _check(load_library().srs_ipc_export(ptr, handle, ctypes.byref(offset)))
        return bytes(handle), int(offset.value)

    def ipc_import(self, handle: bytes) -> int:
        base = ctypes.c_void_p()
        buf = (ctypes.c_char * IPC_HANDLE_BYTES).from_buffer_copy(handle)
        _check(load_library().srs_ipc_import(buf, ctypes.byref(base)))
        return int(base.value)

    def ipc_close(self, base: int) -> None:
        _check(load_library().srs_ipc_close(base))

    def adamw_single(self, row, m_fmt, m_rule, v_fmt, v_rule, hp, stream, grid_ctas=0):
        _check(load_library().srs_adamw_single(ctypes.byref(row), m_fmt, m_rule, v_fmt, v_rule,
                                               ctypes.byref(hp), grid_ctas, stream))

    def sgdm_single(self, row, u_fmt, u_rule, hp, stream, grid_ctas=0):
        _check(load_library().srs_sgdm_single(ctypes.byref(row), u_fmt, u_rule,
                                              ctypes.byref(hp), grid_ctas, stream))

    def derive_keys(self, index_ptr, out_ptr, n, rng, stream):
        _check(load_library().srs_derive_keys(index_ptr, out_ptr, n, ctypes.byref(rng), stream))


_launcher = NativeLauncher()


def launcher():
    return _launcher


def set_launcher(obj):
    """Install a different launcher (tests without a GPU); returns the previous one."""
    global _launcher
    previous, _launcher = _launcher, obj
    return previous
