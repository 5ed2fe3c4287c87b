"""The C ABI without a GPU: every function include/srs_b200.h declares is exported by
libsrs_b200.so, the ctypes mirrors have the C layouts, and invalid arguments are
rejected with an error code and text before any CUDA call."""

import ctypes
import re
import shutil
import subprocess
from pathlib import Path

import pytest

from sr_states.cuda import _native

HEADER = Path(__file__).resolve().parents[1] / "include" / "srs_b200.h"


def declared_functions():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^(?:int|int64_t|const char\*)\s+(srs_\w+)\(", text, re.M)))


def test_every_declared_function_is_exported():
    lib = _native.load_library()
    names = declared_functions()
    assert len(names) >= 10
    for name in names:
        assert hasattr(lib, name), name
    assert set(names) == set(_native._SIGNATURES)


def test_header_constants_match_python():
    text = HEADER.read_text()
    define = dict(re.findall(r"#define\s+(SRS_\w+)\s+\(?(-?(?:0x[0-9A-Fa-f]+|\d+))", text))
    assert int(define["SRS_ABI_VERSION"]) == _native.ABI_VERSION
    assert int(define["SRS_MAX_STEP_CLASSES"]) == _native.MAX_STEP_CLASSES
    assert int(define["SRS_ROW_CLASS_SHIFT"]) == _native.ROW_CLASS_SHIFT
    assert int(define["SRS_ROW_PARAM_BF16"], 16) == _native.ROW_PARAM_BF16
    assert int(define["SRS_ROW_GRAD_BF16"], 16) == _native.ROW_GRAD_BF16
    assert int(define["SRS_ROW_VECTOR_OK"], 16) == _native.ROW_VECTOR_OK
    assert int(define["SRS_ERR_INVALID_ARGUMENT"]) == _native.SRS_ERR_INVALID_ARGUMENT
    assert int(define["SRS_PEERS_STORE"]) == _native.PEERS_STORE
    assert int(define["SRS_PEERS_MULTICAST"]) == _native.PEERS_MULTICAST


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs a C compiler")
def test_struct_layouts_match_ctypes(tmp_path):
    probe = tmp_path / "layout.c"
    probe.write_text(f"""
#include <stddef.h>
#include <stdio.h>
#include "{HEADER}"
int main(void) {{
  printf("%zu %zu %zu %zu\\n", sizeof(srs_row), sizeof(srs_rng), sizeof(srs_adamw_hparams),
         sizeof(srs_sgdm_hparams));
  printf("%zu %zu %zu %zu\\n", offsetof(srs_row, numel), offsetof(srs_row, param_index),
         offsetof(srs_row, flags), offsetof(srs_adamw_hparams, neg_step_size));
  printf("%zu %zu %zu %zu\\n", sizeof(srs_peers), offsetof(srs_peers, mode),
         offsetof(srs_peers, delta_bf16), offsetof(srs_peers, mc_delta_bf16));
  return 0;
}}
""")
    exe = tmp_path / "layout"
    subprocess.run(["gcc", str(probe), "-o", str(exe)], check=True)
    sizes, offsets, peers = subprocess.run([str(exe)], capture_output=True, text=True,
                                           check=True).stdout.split("\n")[:3]
    assert [int(x) for x in peers.split()] == [
        ctypes.sizeof(_native.SrsPeers), _native.SrsPeers.mode.offset,
        _native.SrsPeers.delta_bf16.offset, _native.SrsPeers.mc_delta_bf16.offset]
    assert [int(x) for x in sizes.split()] == [
        ctypes.sizeof(_native.SrsRow), ctypes.sizeof(_native.SrsRng),
        ctypes.sizeof(_native.SrsAdamWHparams), ctypes.sizeof(_native.SrsSgdmHparams)]
    assert [int(x) for x in offsets.split()] == [
        _native.SrsRow.numel.offset, _native.SrsRow.param_index.offset,
        _native.SrsRow.flags.offset, _native.SrsAdamWHparams.neg_step_size.offset]
    assert _native.ROW_DTYPE.itemsize == ctypes.sizeof(_native.SrsRow)
    for field in ("numel", "param_index", "flags"):
        assert _native.ROW_DTYPE.fields[field][1] == getattr(_native.SrsRow, field).offset


def test_library_information_without_a_gpu():
    lib = _native.load_library()
    assert lib.srs_abi_version() == 6
    assert lib.srs_tile_elems() == 2048


def test_invalid_arguments_fail_with_text_and_touch_no_device():
    lib = _native.load_library()
    assert lib.srs_cast(None, None, 0, 9, 0, 0, 0, 0, None) == _native.SRS_ERR_INVALID_ARGUMENT
    assert b"format" in lib.srs_last_error()
    assert lib.srs_cast(None, None, 5, 1, 7, 0, 0, 0, None) == _native.SRS_ERR_INVALID_ARGUMENT
    assert b"rule" in lib.srs_last_error()
    assert lib.srs_cast(None, None, 0, 1, 1, 0, 0, 0, None) == _native.SRS_OK  # empty: no-op
    assert lib.srs_cast(None, None, 4, 1, 1, 0, 0, 0, None) == _native.SRS_ERR_INVALID_ARGUMENT
    hp = _native.SrsAdamWHparams()
    rng = _native.SrsRng()
    hp.n_step_classes = 0
    rc = lib.srs_adamw_multi(None, 0, 0, 1, 1, 1, 1, ctypes.byref(hp), ctypes.byref(rng),
                             _native.KIND_MIXED, 0, None)
    assert rc == _native.SRS_ERR_INVALID_ARGUMENT and b"n_step_classes" in lib.srs_last_error()
    hp.n_step_classes = 1
    rng.key_mode = 5
    rc = lib.srs_adamw_multi(None, 0, 0, 1, 1, 1, 1, ctypes.byref(hp), ctypes.byref(rng), 0, 0,
                             None)
    assert rc == _native.SRS_ERR_INVALID_ARGUMENT and b"key_mode" in lib.srs_last_error()
    rng.key_mode = 0
    rc = lib.srs_adamw_multi(None, 0, 4, 1, 1, 1, 1, ctypes.byref(hp), ctypes.byref(rng), 3, 0,
                             None)
    assert rc == _native.SRS_ERR_INVALID_ARGUMENT and b"without rows" in lib.srs_last_error()
    rc = lib.srs_sgdm_multi(None, 0, 0, 6, 1, None, None, 0, 0, None)
    assert rc == _native.SRS_ERR_INVALID_ARGUMENT
    row = _native.SrsRow()
    row.numel = -1
    rc = lib.srs_sgdm_single(ctypes.byref(row), 1, 1, ctypes.byref(_native.SrsSgdmHparams()), 0,
                             None)
    assert rc == _native.SRS_ERR_INVALID_ARGUMENT and b"negative" in lib.srs_last_error()
    row.numel = 0
    rc = lib.srs_sgdm_single(ctypes.byref(row), 1, 1, ctypes.byref(_native.SrsSgdmHparams()), 0,
                             None)
    assert rc == _native.SRS_OK


def test_native_launcher_refuses_cpu_tensors():
    import torch

    with pytest.raises(ValueError, match="CUDA tensors"):
        _native.NativeLauncher().check_device(torch.device("cpu"))
