"""The library's GGUF reader on good and damaged files (no GPU needed):
s3t_gguf_inspect parses a file exactly as s3t_load_gguf does, so every
count, size and offset read from the file must be checked against its length.
A damaged file must return -1 with a message, never abort the process or
allocate by an unchecked count (the C ABI promises that nothing throws
across it)."""

import ctypes as C
import shutil
import struct

import pytest


@pytest.fixture(scope="module")
def libs3t():
    from sam3cpp_b200 import LIB_PATH, lib
    if not LIB_PATH.exists():
        pytest.skip("libs3t.so not built")
    return lib()


@pytest.fixture(scope="module")
def good(tmp_path_factory):
    from sam3cpp_b200 import synthetic as s
    d = tmp_path_factory.mktemp("gguf")
    return s.write_gguf(d / "one_block.gguf", s.make_f32_weights(0, layers=1), "f16")


def inspect(libs3t, path, map_path=None):
    nt, nl = C.c_int(-1), C.c_int(-1)
    rc = libs3t.s3t_gguf_inspect(str(path).encode(), map_path, C.byref(nt), C.byref(nl))
    return rc, nt.value, nl.value, libs3t.s3t_last_error().decode()


def damaged(good, tmp_path, name, edit):
    p = tmp_path / name
    data = bytearray(good.read_bytes())
    data = edit(data)
    p.write_bytes(bytes(data))
    shutil.copy(str(good) + ".tensor_map.json", str(p) + ".tensor_map.json")
    return p


def test_good_file(libs3t, good):
    rc, nt, nl, _ = inspect(libs3t, good)
    assert (rc, nt, nl) == (0, 16, 1)


def test_missing_file(libs3t, tmp_path):
    rc, *_, msg = inspect(libs3t, tmp_path / "nope.gguf")
    assert rc == -1 and "cannot open" in msg


@pytest.mark.parametrize("case", ["magic", "short", "version", "tensor_count", "kv_count", "header_cut",
                                  "data_cut", "dims"])
def test_damaged_file_is_an_error(libs3t, good, tmp_path, case):
    def set_u64(off, v):
        return lambda d: d[:off] + bytearray(struct.pack("<Q", v)) + d[off + 8:]

    edits = {
        "magic": lambda d: bytearray(b"GGUX") + d[4:],
        "short": lambda d: d[:20],
        "version": lambda d: d[:4] + bytearray(struct.pack("<I", 99)) + d[8:],
        "tensor_count": set_u64(8, 1 << 62),
        "kv_count": set_u64(16, 1 << 62),
        "header_cut": lambda d: d[:200],
        "data_cut": lambda d: d[: len(d) - 4096],
        "dims": None,
    }
    if case == "dims":
        # the first tensor record's dimension count, just after its name
        data = good.read_bytes()
        from sam3cpp_b200 import synthetic as s
        name = s.short_name(s.trunk_tensor_names(1)[0]).encode()
        pos = data.index(struct.pack("<Q", len(name)) + name) + 8 + len(name)
        edits["dims"] = lambda d: d[:pos] + bytearray(struct.pack("<I", 7)) + d[pos + 4:]
    p = damaged(good, tmp_path, f"{case}.gguf", edits[case])
    rc, *_, msg = inspect(libs3t, p)
    assert rc == -1 and msg, case
