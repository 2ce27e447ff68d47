"""The C ABI without a GPU: the library loads, exports every entry point include/foidfinder_b200.h
declares (and the Python signature table covers exactly those), and host-side argument checks return
FF_ERR_INVALID_ARGUMENT with a message before any CUDA call."""

from __future__ import annotations

import ctypes as C
import re
import subprocess
from pathlib import Path

import pytest

from foidfinder_b200 import _lib

ROOT = Path(__file__).resolve().parents[1]
HEADER = (ROOT / "include" / "foidfinder_b200.h").read_text()
DECLARED = sorted(set(re.findall(r"^[A-Za-z_][\w\s\*]*?\b(ff_\w+)\(", HEADER, flags=re.M)))
DEFINES = {k: int(v) for k, v in re.findall(r"#define (FF_\w+) (\d+)", HEADER)}
FAKE = 0x10000  # an aligned address the host checks accept; never dereferenced by the failing calls


def test_header_and_signature_table_agree():
    assert len(DECLARED) >= 20
    assert DECLARED == _lib.exported_symbols()


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    for name in DECLARED:
        assert getattr(lib, name) is not None
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True, check=True)
    exported = {line.split()[-1] for line in out.stdout.splitlines() if " T " in line}
    assert set(DECLARED) <= exported
    # Nothing else of the library's own leaks out of the shared object.
    assert {s for s in exported if s.startswith("ff_")} == set(DECLARED)


def test_status_codes_match():
    assert DEFINES["FF_OK"] == _lib.FF_OK == 0
    for code, text in _lib.STATUS.items():
        assert code in DEFINES.values(), text
    assert DEFINES["FF_EPI_QKV_ROPE"] == _lib.EPI_QKV_ROPE
    assert DEFINES["FF_EPI_RESIDUAL"] == _lib.EPI_RESIDUAL
    assert DEFINES["FF_EPI_SWIGLU"] == _lib.EPI_SWIGLU
    assert DEFINES["FF_EPI_BIAS"] == _lib.EPI_BIAS
    assert DEFINES["FF_EPI_S32"] == _lib.EPI_S32


def test_version():
    assert _lib.lib().ff_version() == 100


def _err() -> str:
    return _lib.lib().ff_last_error().decode()


def test_gemm_rejects_unknown_epilogue():
    rc = _lib.lib().ff_gemm_s8(FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, 128, 128, 128, 99, None, None, 0, 1, 0, None)
    assert rc == DEFINES["FF_ERR_INVALID_ARGUMENT"]
    assert "unknown epilogue 99" in _err()


def test_gemm_rejects_ragged_n():
    rc = _lib.lib().ff_gemm_s8(FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, 128, 100, 128, _lib.EPI_BIAS, None, None, 0, 1, 0, None)
    assert rc == DEFINES["FF_ERR_INVALID_ARGUMENT"]
    assert "multiple of 128" in _err()


def test_gemm_qkv_needs_rope():
    rc = _lib.lib().ff_gemm_s8(FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, 128, 384, 128, _lib.EPI_QKV_ROPE, None, None, 256,
                               1, 0, None)
    assert rc == DEFINES["FF_ERR_INVALID_ARGUMENT"]
    assert "RoPE" in _err()


@pytest.mark.parametrize(
    "args,msg",
    [
        ((None, None, None, 1e-6, 4, 1024, 1024, 1024, FAKE, FAKE, None), "NULL pointer"),
        ((FAKE, None, None, 1e-6, 4, 1000, 1000, 1000, FAKE, FAKE, None), "1000 columns"),
        ((FAKE, FAKE, None, 1e-6, 4, 1024, 1024, 1024, FAKE, FAKE, None), "both"),
        ((FAKE + 2, None, None, 1e-6, 4, 1024, 1024, 1024, FAKE, FAKE, None), "aligned"),
        ((FAKE, None, None, 1e-6, 4, 1024, 1025, 1024, FAKE, FAKE, None), "valid_cols"),
    ],
)
def test_rot_q8_host_checks(args, msg):
    assert _lib.lib().ff_rot_q8(*args) == DEFINES["FF_ERR_INVALID_ARGUMENT"]
    assert msg in _err()


def test_rot_q8_zero_rows_is_a_no_op():
    assert _lib.lib().ff_rot_q8(FAKE, None, None, C.c_float(1e-6), 0, 1024, 1024, 1024, FAKE, FAKE, None) == 0


@pytest.mark.parametrize("seqs,seq_len,heads,rope,msg", [(1, 0, 16, None, "bad shape"), (1, 1025, 65, None, "bad shape"),
                                                     (1, 1025, 16, (FAKE, None), "RoPE tables must be NULL"),
                                                     (1, 1025, 16, (FAKE, FAKE), "RoPE tables must be NULL")])
def test_attention_host_checks(seqs, seq_len, heads, rope, msg):
    cos, sin = rope or (None, None)
    rc = _lib.lib().ff_attention(FAKE, FAKE, seqs, seq_len, heads, cos, sin, 1.0, None)
    assert rc == DEFINES["FF_ERR_INVALID_ARGUMENT"]
    assert msg in _err()


def test_attention_zero_sequences_is_a_no_op():
    assert _lib.lib().ff_attention(FAKE, FAKE, 0, 1025, 16, None, None, 1.0, None) == 0


def test_kernel_error_maps_status():
    with pytest.raises(_lib.KernelError, match="invalid argument"):
        _lib.check(1, "probe")


def test_struct_layouts_match_ctypes(tmp_path):
    """The ctypes mirrors of the header's structs have the C compiler's sizes and field offsets."""
    import shutil

    gcc = shutil.which("gcc") or shutil.which("cc")
    if gcc is None:
        pytest.skip("no C compiler")
    structs = {"ff_model_config": _lib.ModelConfig, "ff_layer_weights": _lib.LayerWeights,
               "ff_model_weights": _lib.ModelWeights}
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "foidfinder_b200.h"', "int main(void) {"]
    for cname, py in structs.items():
        lines.append(f'  printf("{cname} size %zu\\n", sizeof({cname}));')
        for field, _ in py._fields_:
            lines.append(f'  printf("{cname}.{field} %zu\\n", offsetof({cname}, {field}));')
    lines.append("  return 0;\n}")
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run([gcc, "-I", str(ROOT / "include"), str(src), "-o", str(exe)], check=True)
    got = dict(line.rsplit(" ", 1) for line in subprocess.run([str(exe)], capture_output=True, text=True,
                                                              check=True).stdout.splitlines())
    for cname, py in structs.items():
        assert int(got[f"{cname} size"]) == C.sizeof(py), cname
        for field, _ in py._fields_:
            assert int(got[f"{cname}.{field}"]) == getattr(py, field).offset, f"{cname}.{field}"


def test_pair_tiles_need_int8_and_256_columns():
    pair = DEFINES["FF_TILE_PAIR256"]
    rc = _lib.lib().ff_gemm_s8(FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, 512, 384, 128, _lib.EPI_BIAS, None, None, 0, 1, pair,
                               None)
    assert rc == DEFINES["FF_ERR_INVALID_ARGUMENT"]
    assert "pair tiles" in _err() or "multiple of the tile width" in _err()
    rc = _lib.lib().ff_gemm_f16(FAKE, FAKE, FAKE, FAKE, 512, 256, 128, _lib.EPI_BIAS, 256, 256, None, 0, 0, pair, None)
    assert rc == DEFINES["FF_ERR_INVALID_ARGUMENT"]
    assert "pair tiles need int8" in _err()


@pytest.mark.parametrize(("name", "launches"), [("eva02-l-448", 3 + 9 * 24 + 1 + 1 + 1),
                                                 ("eva02-b-448", 3 + 9 * 12 + 7 + 1 + 1),
                                                 ("pixai-1008", 3 + 9 * 32 + 4 + 1 + 1)])
def test_launches_per_forward(name, launches):
    """Kernel launches of one forward: 9 per block (EVA02's 1025th query row and key are computed inside the
    attention launch), the head's launches, the tag GEMM and the top-k."""
    from foidfinder_b200.config import CONFIGS
    from foidfinder_b200.engine import c_config

    cfg = c_config(CONFIGS[name])
    assert _lib.lib().ff_engine_launches_per_forward(C.byref(cfg)) == launches
