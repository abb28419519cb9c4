"""CPU tests of the .qora-tts reader/writer (save.rs:23-137, 262-409) in
libqtts_b200.so and of the C-ABI surface.  No GPU needed."""
import os
import re
import struct

import numpy as np
import pytest

from conftest import REPO


def test_writer_matches_oracle_writer(qtts, oracle_mod, tmp_path):
    a = str(tmp_path / "prod.qtts")
    b = str(tmp_path / "orc.qtts")
    qtts.synth_write(a, qtts.dims_tiny(), 5)
    oracle_mod.synth_write(b, oracle_mod.dims_tiny(), 5)
    assert open(a, "rb").read() == open(b, "rb").read()


def test_probe_reads_dims(qtts, tiny_path):
    d = qtts.file_probe(tiny_path).as_dict()
    ref = qtts.dims_tiny().as_dict()
    assert d == ref


def test_1p7b_dims_match_config(qtts, oracle_mod):
    d = qtts.dims_1p7b().as_dict()
    o = oracle_mod.dims_1p7b()
    assert d["t_layers"] == 28 and d["t_hidden"] == 2048 and d["t_heads"] == 16 and d["t_kv_heads"] == 8
    assert d["t_inter"] == 6144 and d["t_vocab"] == 3072 and d["p_layers"] == 5 and d["p_hidden"] == 1024
    assert d["p_groups"] == 15 and d["t_sec"] == [24, 20, 20]
    for f, _ in o._fields_:
        if f != "t_sec":
            assert getattr(o, f) == d[f], f


def test_oracle_reads_product_file(oracle_mod, tiny_path):
    m = oracle_mod.Model(tiny_path)
    assert m.dims.t_layers == 2 and m.dims.p_groups == 15
    m.close()


def _corrupt(src, dst, offset, payload):
    data = bytearray(open(src, "rb").read())
    data[offset:offset + len(payload)] = payload
    open(dst, "wb").write(bytes(data))


def test_rejects_bad_magic(qtts, oracle_mod, tiny_path, tmp_path):
    p = str(tmp_path / "bad.qtts")
    _corrupt(tiny_path, p, 0, b"XTTS")
    with pytest.raises(qtts.QttsError) as e:
        qtts.file_probe(p)
    assert e.value.code == qtts.ERR_FORMAT and "magic" in str(e.value)
    with pytest.raises(IOError):
        oracle_mod.Model(p)


def test_rejects_bad_version_and_format(qtts, tiny_path, tmp_path):
    p = str(tmp_path / "v2.qtts")
    _corrupt(tiny_path, p, 4, struct.pack("<I", 2))
    with pytest.raises(qtts.QttsError) as e:
        qtts.file_probe(p)
    assert e.value.code == qtts.ERR_FORMAT
    _corrupt(tiny_path, p, 8, b"\x07")
    with pytest.raises(qtts.QttsError) as e:
        qtts.file_probe(p)
    assert e.value.code == qtts.ERR_FORMAT


def test_rejects_truncated(qtts, tiny_path, tmp_path):
    data = open(tiny_path, "rb").read()
    for cut in (3, 40, len(data) // 2, len(data) - 200):
        p = str(tmp_path / f"trunc{cut}.qtts")
        open(p, "wb").write(data[:cut])
        with pytest.raises(qtts.QttsError) as e:
            qtts.file_probe(p)
        assert e.value.code == qtts.ERR_FORMAT


def test_rejects_weight_length_mismatch(qtts, tiny_path, tmp_path):
    # first Weight record starts after the 9-byte header and 11 u32 talker fields
    off = 9 + 11 * 4
    p = str(tmp_path / "len.qtts")
    _corrupt(tiny_path, p, off + 16, struct.pack("<Q", 12345))  # packed length
    with pytest.raises(qtts.QttsError) as e:
        qtts.file_probe(p)
    assert e.value.code == qtts.ERR_FORMAT
    _corrupt(tiny_path, p, off, struct.pack("<Q", 513))  # q_proj k != hidden
    with pytest.raises(qtts.QttsError) as e:
        qtts.file_probe(p)
    assert e.value.code == qtts.ERR_FORMAT


def test_missing_file(qtts, tmp_path):
    with pytest.raises(qtts.QttsError) as e:
        qtts.file_probe(str(tmp_path / "nope.qtts"))
    assert e.value.code == qtts.ERR_IO


def test_library_exports_every_declared_symbol(qtts):
    header = open(os.path.join(REPO, "include", "qtts.h")).read()
    declared = set(re.findall(r"QTTS_API[^;(]*?\b(qtts_\w+)\s*\(", header))
    assert len(declared) >= 30
    for name in sorted(declared):
        assert hasattr(qtts.lib, name), name
    exported = os.popen(f"nm -D --defined-only {qtts.LIB_PATH}").read()
    for name in declared:
        assert re.search(rf"\b{name}\b", exported), name


def test_bad_arguments_fail_cleanly_without_gpu(qtts):
    import ctypes as C
    h = C.c_void_p()
    rc = qtts.lib.qtts_model_load(b"/nonexistent/model.qtts", 0, C.byref(h))
    assert rc == qtts.ERR_IO
    assert qtts.lib.qtts_q4_gemv_scratch_bytes(0, 32, 1) == 0
    rc = qtts.lib.qtts_q4_gemv(None, None, 8, 32, None, 1, None)
    assert rc == qtts.ERR_BADARG
    x = np.zeros(4, np.float32)
    assert qtts.lib.qtts_generate_frames(None, 1) == qtts.ERR_BADARG
    del x


def test_quantize_arguments_rejected_on_the_host(qtts):
    # gemv.rs:92-130 needs n % 32 == 0; these are refused before any CUDA call
    with pytest.raises(qtts.QttsError) as e:
        qtts.quantize_f32_to_q4(np.zeros((2, 48), np.float32), 2, 48)
    assert e.value.code == qtts.ERR_BADARG
    with pytest.raises(qtts.QttsError) as e:
        qtts.quantize_f32_to_q4(np.zeros((2, 64), np.float32), 3, 64)  # size mismatch
    assert e.value.code == qtts.ERR_BADARG
    assert qtts.lib.qtts_q4_quantize(None, 2, 64, None, None) == qtts.ERR_BADARG
    assert qtts.lib.qtts_q4_quantize_dev(None, 2, 64, None, None, None) == qtts.ERR_BADARG
