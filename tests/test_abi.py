"""CPU: the C-ABI library loads, exports every symbol include/tidegs_b200.h
declares, and validates arguments on the host (no kernel launches here)."""
import ctypes
import re
from pathlib import Path

import pytest

from tidegs_b200 import _lib

HEADER = Path(__file__).resolve().parent.parent / "include" / "tidegs_b200.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^TGS_API\s+[\w\s\*]+?\b(tgs_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_the_entry_points():
    syms = declared_symbols()
    assert "tgs_resident_adam_apply" in syms and "tgs_pack_rows" in syms
    assert len(syms) >= 19


def test_library_loads_and_exports_every_declared_symbol():
    lib = _lib.load()
    for name in declared_symbols():
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"
    assert lib.tgs_version() == _lib.ABI_VERSION


def test_bindings_cover_only_declared_symbols():
    assert set(_lib.SIGNATURES) <= set(declared_symbols())


def test_null_args_are_rejected_with_a_message():
    lib = _lib.load()
    assert lib.tgs_resident_adam_count(None, None) == 1
    assert "NULL" in _lib.last_error()
    assert lib.tgs_unpack_rows(None, None) == 1
    with pytest.raises(RuntimeError, match="tgs_copy_blocks"):
        _lib.call("tgs_copy_blocks", None, None)


def test_empty_work_is_a_no_op_without_device():
    lib = _lib.load()
    args = _lib.DenseArgs()
    args.n_groups = 0
    args.n_rows = 0
    assert lib.tgs_selective_adam(ctypes.byref(args), None) == 0
    assert lib.tgs_fill_global_ids(None, 0, None, 0, 4, None) == 0
    assert lib.tgs_block_bounds(None, None, None, 0, None, None) == 0
    assert lib.tgs_compact_scratch_words(0) == 1
    assert lib.tgs_compact_scratch_words(2049) == 3
    sh = _lib.ShArgs()
    sh.n, sh.K, sh.degree = 0, 16, 3
    assert lib.tgs_sh_fwd(ctypes.byref(sh), None) == 0
    assert lib.tgs_isect_depth_order(None, None, 0, None, None, None, 0, None) == 0
    assert lib.tgs_isect_expand_ids(None, 2, None, None, 0, None, None) == 0


def test_render_argument_checks_without_device():
    lib = _lib.load()
    sh = _lib.ShArgs()
    sh.n, sh.K, sh.degree = 5, 9, 3  # degree 3 needs 16 coefficients
    assert lib.tgs_sh_fwd(ctypes.byref(sh), None) == 1
    assert "degree 3" in _lib.last_error()
    sh.K, sh.degree = 26, 4  # at most 25 coefficients
    assert lib.tgs_sh_fwd(ctypes.byref(sh), None) == 1
    # key widths: 13 bits (one camera, 120 x 68 tiles) fit 16-bit keys; 70
    # cameras at 4K (240 x 135 tiles) need 32-bit keys; beyond 32 bits: none
    assert lib.tgs_isect_key_bytes(1, 120, 68) == 2
    assert lib.tgs_isect_key_bytes(70, 240, 135) == 4
    assert lib.tgs_isect_key_bytes(65535, 65535, 2) == 0
    assert lib.tgs_isect_sort_tiles(None, None, 10, 65535, 65535, 2, None, None, None, 0,
                                    None) == 1
    assert lib.tgs_isect_tile_bits(8160) == 13


def test_struct_layouts_match_the_header_sizes():
    # field counts mirror the C structs; offsets follow the platform C ABI
    assert ctypes.sizeof(_lib.DenseGroup) == 5 * 8 + 8 + 6 * 4
    assert ctypes.sizeof(_lib.DenseArgs) == 16 * ctypes.sizeof(_lib.DenseGroup) + 8 + 8 + 8 + 8
    assert _lib.ResidentAdamArgs.lr.offset == 96
    assert _lib.ResidentAdamArgs.batch_size.offset == 96 + 24 + 5 * 4


def test_struct_offsets_match_the_c_compiler(tmp_path):
    """Every field offset and struct size of the ctypes mirrors equals what a
    C compiler computes from include/tidegs_b200.h."""
    import shutil
    import subprocess
    from pathlib import Path

    if shutil.which("gcc") is None:
        pytest.skip("gcc not available")
    structs = {name: getattr(_lib, name) for name in (
        "ResidentCountArgs", "ResidentAdamArgs", "DenseGroup", "DenseArgs", "UnpackArgs",
        "CopyBlocksArgs", "PackArgs", "BlockSumArgs", "GradPushArgs", "PeerHandle",
        "ResidentAdamSumArgs", "SparseAccumArgs", "CullArgs", "ProjectArgs",
        "ProjectBwdArgs", "RasterArgs", "RasterBwdArgs", "ShArgs", "ShBwdArgs")}
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "tidegs_b200.h"',
             'int main(void) {']
    expect = []
    for name, cls in structs.items():
        c_name = "Tgs" + name
        lines.append(f'  printf("%zu\\n", sizeof({c_name}));')
        expect.append(ctypes.sizeof(cls))
        for field, _ in cls._fields_:
            lines.append(f'  printf("%zu\\n", offsetof({c_name}, {field}));')
            expect.append(getattr(cls, field).offset)
    lines += ["  return 0;", "}"]
    src = tmp_path / "offsets.c"
    src.write_text("\n".join(lines))
    include = Path(__file__).resolve().parents[1] / "include"
    exe = tmp_path / "offsets"
    subprocess.run(["gcc", "-std=c11", f"-I{include}", str(src), "-o", str(exe)], check=True)
    got = [int(x) for x in subprocess.run([str(exe)], check=True, capture_output=True,
                                          text=True).stdout.split()]
    assert got == expect


def test_no_cpu_fallback_without_cuda():
    import torch

    if torch.cuda.is_available():
        pytest.skip("CUDA present")
    from tidegs_b200 import GPUResidentAdam

    with pytest.raises(RuntimeError, match="CUDA"):
        GPUResidentAdam(device="cuda")
    with pytest.raises(RuntimeError, match="no CPU path"):
        GPUResidentAdam(device="cpu")


def test_nvtx_ranges_wrap_calls_when_enabled(monkeypatch):
    calls = []
    monkeypatch.setattr(_lib, "NVTX", True)
    import torch

    monkeypatch.setattr(torch.cuda.nvtx, "range_push", lambda n: calls.append(("push", n)))
    monkeypatch.setattr(torch.cuda.nvtx, "range_pop", lambda: calls.append(("pop",)))
    _lib.call("tgs_fill_global_ids", None, 0, None, 0, 4, None)  # no work: no device needed
    with pytest.raises(RuntimeError, match="tgs_copy_blocks"):
        _lib.call("tgs_copy_blocks", None, None)
    assert calls == [("push", "tgs_fill_global_ids"), ("pop",), ("push", "tgs_copy_blocks"),
                     ("pop",)]

