"""C ABI checks that need no GPU: the library loads, exports every symbol that
include/*.h declares, and the reference's NULL-safety / error conventions hold
(src/voicedetect_capi.cpp:61-176; tests/test_smoke.cpp in the reference checks
the version and ABI number)."""
import ctypes as C
import re
from pathlib import Path

import pytest

import vd_b200

ROOT = Path(__file__).resolve().parents[1]


def _declared_functions():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        text = re.sub(r"//.*", "", text)
        for m in re.finditer(r"\b((?:voicedetect|vdb)_[a-z0-9_]+)\s*\(", text):
            names.add(m.group(1))
    return sorted(names)


def test_library_exports_every_declared_symbol():
    L = C.CDLL(str(vd_b200.LIB_PATH))
    names = _declared_functions()
    assert len(names) >= 25
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing


def test_abi_version_and_null_safety():
    L = vd_b200.lib()
    assert L.voicedetect_capi_abi_version() == 1
    assert L.voicedetect_capi_last_error(None) == b""
    L.voicedetect_capi_free(None)
    L.voicedetect_capi_free_vec(None)
    L.voicedetect_capi_free_string(None)
    assert L.voicedetect_capi_load(None) is None
    assert L.voicedetect_capi_load(b"/nonexistent/model.gguf") is None
    # every model call on a NULL context reports an error, never crashes
    p = C.POINTER(C.c_float)()
    d = C.c_int(7)
    assert L.voicedetect_capi_embed_path(None, b"x.wav", C.byref(p), C.byref(d)) == 1
    assert not p and d.value == 0  # outputs reset before work
    assert L.voicedetect_capi_verify_paths(None, b"a", b"b", 0.25, None, None) == 1
    assert L.voicedetect_capi_analyze_path_json(None, b"a") is None
    assert L.voicedetect_capi_set_devices(None, 1) == 1
    # the page-locking helpers refuse NULL / empty ranges before touching CUDA
    assert L.voicedetect_b200_host_register(None, 16) == 1
    assert b"NULL" in L.vdb_last_error()
    assert L.voicedetect_b200_host_unregister(None) == 1


def test_load_rejects_corrupt_gguf(tmp_path):
    import vd_synth
    L = vd_b200.lib()
    good = tmp_path / "m.gguf"
    vd_synth.write_resnet_gguf(str(good), vd_synth.tiny_resnet_model(1, n_mels=16))
    data = good.read_bytes()
    bad_magic = tmp_path / "bad_magic.gguf"
    bad_magic.write_bytes(b"XXXX" + data[4:])
    truncated = tmp_path / "trunc.gguf"
    truncated.write_bytes(data[: len(data) // 2])
    empty = tmp_path / "empty.gguf"
    empty.write_bytes(b"")
    missing = tmp_path / "missing.gguf"
    # a directory cannot be mapped or read: the loader's plain-read fallback must fail
    for p in (bad_magic, truncated, empty, missing, tmp_path):
        assert L.voicedetect_capi_load(str(p).encode()) is None


def test_op_entry_points_reject_bad_arguments():
    L = vd_b200.lib()
    assert L.vdb_conv(None, None) != 0
    assert b"NULL" in L.vdb_last_error()
    a = vd_b200.ConvArgs(batch=1, t_out=4, f_out=4, oc=24, k0=3, stride0=1, ic0=32)
    assert L.vdb_conv(C.byref(a), None) != 0  # oc not a multiple of 16
    assert L.vdb_fbank_plan_create(16000, 80, 400, 400, 160, 0.97, 20.0, 0.0) is None
    assert L.vdb_identify(None, 1, None, 1, 1, 1, None, None, None) != 0
    assert L.vdb_grid_rows(2, 10, 8) == 2 * 12 * 10
    assert L.vdb_phase_rows(2, 10, 8) == 4 * 2 * 7 * 6


def _tensor_table_dims(data: bytes):
    """Byte offsets of every tensor's dimension fields in a GGUF v2/v3 file
    (the tensor-info table that follows the metadata)."""
    import struct
    pos = 8
    n_t, n_kv = struct.unpack_from("<QQ", data, pos)
    pos += 16
    sizes = {0: 1, 1: 1, 2: 2, 3: 2, 4: 4, 5: 4, 6: 4, 7: 1, 10: 8, 11: 8, 12: 8}

    def skip_str(p):
        (n,) = struct.unpack_from("<Q", data, p)
        return p + 8 + n

    def skip_val(p, t):
        if t == 8:
            return skip_str(p)
        if t == 9:
            at, n = struct.unpack_from("<IQ", data, p)
            p += 12
            for _ in range(n):
                p = skip_val(p, at)
            return p
        return p + sizes[t]

    for _ in range(n_kv):
        pos = skip_str(pos)
        (t,) = struct.unpack_from("<I", data, pos)
        pos = skip_val(pos + 4, t)
    out = []
    for _ in range(n_t):
        pos = skip_str(pos)
        (nd,) = struct.unpack_from("<I", data, pos)
        pos += 4
        out.append((nd, pos))
        pos += 8 * nd + 4 + 8
    return out


def test_load_rejects_overflowing_tensor_dimensions(tmp_path, capfd):
    """A tensor whose dimensions multiply past 2^64 (so the byte count would wrap to
    a small value) is refused at load instead of passing the bounds check."""
    import struct

    import vd_synth
    L = vd_b200.lib()
    good = tmp_path / "m.gguf"
    vd_synth.write_resnet_gguf(str(good), vd_synth.tiny_resnet_model(1, n_mels=16))
    data = bytearray(good.read_bytes())
    dims = _tensor_table_dims(bytes(data))
    nd, pos = next((nd, p) for nd, p in dims if nd == 4)
    ne = list(struct.unpack_from("<4Q", data, pos))
    # 2^62 * 2^2 * ... : every product wraps modulo 2^64
    cases = [[ne[0], 1 << 62, 4, 1 << 33], [ne[0], ne[1], 1 << 40, 1 << 40],
             [1 << 63, 1, 1, 1]]
    for k, bad_ne in enumerate(cases):
        bad = bytearray(data)
        struct.pack_into("<4Q", bad, pos, *bad_ne)
        p = tmp_path / f"overflow{k}.gguf"
        p.write_bytes(bytes(bad))
        assert L.voicedetect_capi_load(str(p).encode()) is None
        err = capfd.readouterr().err
        if bad_ne[0] >= 1 << 63:  # negative as int64
            assert "non-positive dimension" in err, err
        else:
            assert "larger than the file" in err, err
