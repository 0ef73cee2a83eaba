"""CPU: expert loading from files. The expert store (include/moert_store.h) against the reference's
own store code (moert/memmgr/store.cpp, built into oracle/_ref): identical files for identical
pages, each side reading the other's, checksum verification; the GGUF fixture writer against the
reference's gguf_write_to_file; the library's GGUF directory and type sizes against ggml's; and a
layer round trip GGUF + store -> load_host_layer."""
import ctypes as C
import os

import numpy as np
import pytest

from conftest import ROOT, host_layer
from gguf_fixture import F32, STR, U32, layer_files, write_gguf

REF_STORE = os.path.join(ROOT, "oracle", "_ref", "libmoert_store_ref.so")
REF_GGML = os.path.join(ROOT, "oracle", "_ref", "libggml_ref.so")
STORE_FNS = [n for n in ("moert_store_probe", "moert_store_verify", "moert_store_writer_open",
                         "moert_store_writer_add_page", "moert_store_writer_close", "moert_store_fnv1a64",
                         "moert_store_reader_open", "moert_store_reader_free", "moert_store_reader_geometry",
                         "moert_store_reader_page_nbytes", "moert_store_reader_page_info", "moert_store_reader_read")]


@pytest.fixture(scope="module")
def ours():
    from llapis_b200 import capi
    return capi.lib()


@pytest.fixture(scope="module")
def ref_store():
    if not os.path.exists(REF_STORE):
        pytest.skip("oracle/_ref/libmoert_store_ref.so not built (make -C oracle ref)")
    from llapis_b200 import capi
    lib = C.CDLL(REF_STORE)
    for n in STORE_FNS:
        res, args = capi.SIGNATURES[n]
        getattr(lib, n).restype, getattr(lib, n).argtypes = res, args
    return lib


def pages(seed=3, n_expert=6, n_layers=2):
    rng = np.random.default_rng(seed)
    out = []
    for layer in range(n_layers):
        for e in range(0, n_expert, 2):   # every other expert, both kinds, plus a scale page
            out.append(dict(layer=layer, expert=e, kind=0, is_scale=0, quant_type=12, source_quant=12, flags=0,
                            shape=(512, 128), data=rng.integers(0, 256, 1000 + 37 * e, dtype=np.uint8)))
            out.append(dict(layer=layer, expert=e, kind=1, is_scale=0, quant_type=6, source_quant=20, flags=2,
                            shape=(64, 512), data=rng.integers(0, 256, 700, dtype=np.uint8)))
            out.append(dict(layer=layer, expert=e, kind=1, is_scale=1, quant_type=0, source_quant=0, flags=0,
                            shape=(1,), data=np.array([0.5 + e], np.float32).view(np.uint8)))
    return out


def write_with(lib, index, pack, pg, n_layers=2, n_expert=6, pack_uuid=0x1234, source_uuid=77):
    from llapis_b200 import capi
    info = capi.StoreInfo(0, source_uuid, b"gemma4", n_layers, n_expert, 512, 64, pack_uuid, 0)
    w = lib.moert_store_writer_open(index.encode(), pack.encode(), C.byref(info))
    assert w
    for p in pg:
        d = np.ascontiguousarray(p["data"])
        assert lib.moert_store_writer_add_page(w, p["layer"], p["expert"], p["kind"], p["is_scale"], p["quant_type"],
                                               p["source_quant"], p["flags"], (C.c_int64 * 4)(*p["shape"]),
                                               len(p["shape"]), d.ctypes.data, d.size) == 1
    assert lib.moert_store_writer_close(w) == 1


def read_all(lib, index, pg):
    r = lib.moert_store_reader_open(index.encode(), 0)
    assert r
    try:
        nl, ne = C.c_int32(), C.c_int32()
        assert lib.moert_store_reader_geometry(r, C.byref(nl), C.byref(ne)) == 1 and (nl.value, ne.value) == (2, 6)
        for p in pg:
            buf = np.zeros(p["data"].size + 8, np.uint8)
            got = lib.moert_store_reader_read(r, p["layer"], p["kind"], p["is_scale"], p["expert"], buf.ctypes.data,
                                              buf.size, 1)
            assert got == p["data"].size and np.array_equal(buf[:got], p["data"])
            qt, nb, shape = C.c_int32(), C.c_uint64(), (C.c_int64 * 4)()
            assert lib.moert_store_reader_page_info(r, p["layer"], p["kind"], p["is_scale"], p["expert"], C.byref(qt),
                                                    C.byref(nb), shape) == 1
            assert (qt.value, nb.value) == (p["quant_type"], p["data"].size)
            assert list(shape) == list(p["shape"]) + [1] * (4 - len(p["shape"]))
        # absent pages: an odd expert, a kind with no pages, a kind outside 0..3, a layer out of range
        for args in ((0, 0, 0, 1), (0, 2, 0, 0), (0, 5, 0, 0), (2, 0, 0, 0), (0, 0, 1, 0)):
            assert lib.moert_store_reader_page_nbytes(r, *args) == 0
        small = np.zeros(10, np.uint8)   # a destination that is too small reads nothing
        assert lib.moert_store_reader_read(r, 0, 0, 0, 0, small.ctypes.data, small.size, 0) == 0
    finally:
        lib.moert_store_reader_free(r)


def test_fnv1a64_matches_reference(ours, ref_store):
    rng = np.random.default_rng(1)
    for n in (0, 1, 7, 4096):
        d = rng.integers(0, 256, n, dtype=np.uint8)
        for seed in (14695981039346656037, 12345):
            assert ours.moert_store_fnv1a64(d.ctypes.data, n, seed) == ref_store.moert_store_fnv1a64(d.ctypes.data, n, seed)


def test_store_files_identical_to_reference(ours, ref_store, tmp_path):
    pg = pages()
    a, b = str(tmp_path / "a.experts.index"), str(tmp_path / "b.experts.index")
    write_with(ours, a, a.replace("index", "pack"), pg)
    write_with(ref_store, b, b.replace("index", "pack"), pg)
    for x, y in ((a, b), (a.replace("index", "pack"), b.replace("index", "pack"))):
        assert open(x, "rb").read() == open(y, "rb").read()


def test_store_cross_read_and_verify(ours, ref_store, tmp_path):
    from llapis_b200 import capi
    pg = pages(seed=9)
    for writer, name in ((ours, "o"), (ref_store, "r")):
        idx = str(tmp_path / f"{name}.experts.index")
        write_with(writer, idx, idx.replace("index", "pack"), pg)
        for reader in (ours, ref_store):
            read_all(reader, idx, pg)
            assert reader.moert_store_verify(idx.encode()) == 0
            info = capi.StoreInfo()
            assert reader.moert_store_probe(idx.encode(), C.byref(info)) == 1
            assert (info.n_layers, info.n_expert, info.record_count, info.pack_uuid, info.source_uuid,
                    info.arch) == (2, 6, len(pg), 0x1234, 77, b"gemma4")
            assert not reader.moert_store_reader_open(idx.encode(), 78)      # another source's store
        # one flipped byte in one page: both verifiers count exactly one bad page
        pack = idx.replace("index", "pack")
        raw = bytearray(open(pack, "rb").read())
        raw[256 + 5] ^= 0xFF   # inside the first page (pages start on 256-byte boundaries)
        open(pack, "wb").write(bytes(raw))
        assert ours.moert_store_verify(idx.encode()) == 1 and ref_store.moert_store_verify(idx.encode()) == 1


def test_store_writer_rejects_bad_pages(ours, ref_store, tmp_path):
    for lib, name in ((ours, "o"), (ref_store, "r")):
        idx = str(tmp_path / f"{name}.experts.index")
        from llapis_b200 import capi
        info = capi.StoreInfo(0, 1, b"gemma4", 1, 4, 0, 0, 5, 0)
        w = lib.moert_store_writer_open(idx.encode(), idx.replace("index", "pack").encode(), C.byref(info))
        d = np.zeros(16, np.uint8)
        assert lib.moert_store_writer_add_page(w, 0, 9, 0, 0, 12, 12, 0, (C.c_int64 * 4)(1, 1, 1, 1), 1,
                                               d.ctypes.data, d.size) == 0   # expert out of range
        assert lib.moert_store_writer_close(w) == 0
        assert not os.path.exists(idx)


@pytest.fixture(scope="module")
def ref_ggml():
    if not os.path.exists(REF_GGML):
        pytest.skip("oracle/_ref/libggml_ref.so not built")
    lib = C.CDLL(REF_GGML)

    class Params(C.Structure):
        _fields_ = [("mem_size", C.c_size_t), ("mem_buffer", C.c_void_p), ("no_alloc", C.c_bool)]
    lib.Params = Params
    for n, res, args in (("ggml_init", C.c_void_p, [Params]), ("ggml_free", None, [C.c_void_p]),
                         ("ggml_new_tensor", C.c_void_p, [C.c_void_p, C.c_int, C.c_int, C.POINTER(C.c_int64)]),
                         ("ggml_set_name", C.c_void_p, [C.c_void_p, C.c_char_p]),
                         ("ggml_get_data", C.c_void_p, [C.c_void_p]),
                         ("ggml_type_size", C.c_size_t, [C.c_int]), ("ggml_blck_size", C.c_int64, [C.c_int]),
                         ("gguf_init_empty", C.c_void_p, []), ("gguf_free", None, [C.c_void_p]),
                         ("gguf_set_val_u32", None, [C.c_void_p, C.c_char_p, C.c_uint32]),
                         ("gguf_set_val_f32", None, [C.c_void_p, C.c_char_p, C.c_float]),
                         ("gguf_set_val_str", None, [C.c_void_p, C.c_char_p, C.c_char_p]),
                         ("gguf_add_tensor", None, [C.c_void_p, C.c_void_p]),
                         ("gguf_write_to_file", C.c_bool, [C.c_void_p, C.c_char_p, C.c_bool])):
        getattr(lib, n).restype, getattr(lib, n).argtypes = res, args
    return lib


def ref_write_gguf(lib, path, kvs, tensors):
    ctx = lib.ggml_init(lib.Params(64 << 20, None, False))
    g = lib.gguf_init_empty()
    try:
        for key, t, v in kvs:
            {U32: lib.gguf_set_val_u32, F32: lib.gguf_set_val_f32,
             STR: lambda c, k, x: lib.gguf_set_val_str(c, k, x.encode())}[t](g, key.encode(), v)
        for name, typ, ne, data in tensors:
            t = lib.ggml_new_tensor(ctx, typ, len(ne), (C.c_int64 * len(ne))(*ne))
            lib.ggml_set_name(t, name.encode())
            C.memmove(lib.ggml_get_data(t), bytes(data), len(data))
            lib.gguf_add_tensor(g, t)
        assert lib.gguf_write_to_file(g, path.encode(), False)
    finally:
        lib.gguf_free(g)
        lib.ggml_free(ctx)


def small_gguf_content():
    rng = np.random.default_rng(4)
    kvs = [("general.architecture", STR, "gemma4"), ("gemma4.expert_count", U32, 4),
           ("gemma4.attention.layer_norm_rms_epsilon", F32, 1e-6)]
    tensors = [("a.weight", 0, (8, 3), rng.standard_normal(24).astype(np.float32).tobytes()),
               ("b.q4k", 12, (256, 2, 4), rng.integers(0, 256, 144 * 8, dtype=np.uint8).tobytes()),
               ("c.iq4nl", 20, (64, 5), rng.integers(0, 256, 18 * 2 * 5, dtype=np.uint8).tobytes())]
    return kvs, tensors


def test_gguf_fixture_writer_matches_reference(ref_ggml, tmp_path):
    kvs, tensors = small_gguf_content()
    a, b = str(tmp_path / "ours.gguf"), str(tmp_path / "ref.gguf")
    write_gguf(a, kvs, tensors)
    ref_write_gguf(ref_ggml, b, kvs, tensors)
    assert open(a, "rb").read() == open(b, "rb").read()


def test_gguf_directory(tmp_path):
    from llapis_b200.loader import Gguf
    kvs, tensors = small_gguf_content()
    p = str(tmp_path / "x.gguf")
    write_gguf(p, kvs, tensors)
    g = Gguf(p)
    assert g.str("general.architecture") == "gemma4" and g.u32("gemma4.expert_count") == 4
    assert g.f32("gemma4.attention.layer_norm_rms_epsilon") == np.float32(1e-6)
    assert g.u32("missing.key") is None and g.tensor("nope") is None
    for name, typ, ne, data in tensors:
        t = g.tensor(name)
        assert (t.type, t.n_dims, tuple(t.ne[:len(ne)]), t.nbytes) == (typ, len(ne), ne, len(data))
        assert t.offset % 32 == 0 and g.read(name).tobytes() == data
    g.close()
    bad = str(tmp_path / "bad.gguf")
    open(bad, "wb").write(b"GGUX" + bytes(32))
    with pytest.raises(Exception):
        Gguf(bad)


def test_type_sizes_match_ggml(ref_ggml, ours, tmp_path):
    """The directory's block sizes (for a tensor's byte count) against ggml's type traits."""
    from llapis_b200.loader import Gguf
    for t in [0, 1, 2, 3, 6, 7, 8, 9, 10, 11, 12, 13, 14, 15, 16, 17, 18, 19, 20, 21, 22, 23, 24, 25, 26, 27, 28, 29, 30]:
        blck, size = int(ref_ggml.ggml_blck_size(t)), int(ref_ggml.ggml_type_size(t))
        p = str(tmp_path / f"t{t}.gguf")
        write_gguf(p, [], [("x", t, (blck * 2, 3), bytes(size * 6))])
        assert Gguf(p).tensor("x").nbytes == size * 6, f"type {t}"


@pytest.mark.parametrize("split", [False, True])
def test_layer_round_trip(tmp_path, split):
    """A layer written as GGUF + store and read back equals the layer it was written from."""
    from llapis_b200 import workload
    from llapis_b200.loader import load_host_layer
    host = host_layer("mini_mixed")
    norms = workload.block_norms(workload.CONFIGS["mini_mixed"])
    gp, sp = str(tmp_path / "m.gguf"), str(tmp_path / "m.gguf.experts.index")
    layer_files(host, norms, gp, sp, il=3, n_layers=4, split_gate_up=split)
    got, gn = load_host_layer(gp, 3, sp, host.hot_ids)
    assert host.b_router is not None   # the mini workload's router bias travels as ffn_gate_inp.bias
    for n in ("w_router", "b_router", "hot_ids", "hot_gu", "hot_down", "cold_gu", "cold_down", "s_hot", "s_cold"):
        a, b = getattr(got, n), getattr(host, n)
        assert (a is None) == (b is None) and (a is None or np.array_equal(np.asarray(a).reshape(-1).view(np.uint8),
                                                                            np.asarray(b).reshape(-1).view(np.uint8))), n
    assert (got.hot_type_gu, got.hot_type_down, got.cold_type_gu, got.cold_type_down, got.top_k) == \
        (host.hot_type_gu, host.hot_type_down, host.cold_type_gu, host.cold_type_down, host.top_k)
    for n in ("pre_norm", "router_scale", "post_norm"):
        assert np.array_equal(getattr(gn, n), getattr(norms, n))
    assert gn.eps == np.float32(1e-6)
    with pytest.raises(Exception):
        load_host_layer(gp, 2, sp, host.hot_ids)   # no such layer in the file


def test_gguf_rejects_malformed_files(tmp_path):
    """Truncated headers, an unknown tensor type, a row that is not whole blocks and data past the
    end of the file all fail to open with a message, and never read past the file."""
    from llapis_b200 import capi
    from llapis_b200.loader import Gguf
    lib = capi.lib()
    kvs, tensors = small_gguf_content()
    good = str(tmp_path / "good.gguf")
    write_gguf(good, kvs, tensors)
    raw = open(good, "rb").read()
    cases = {
        "truncated_header": raw[:20],
        "truncated_infos": raw[:200],
        "data_past_end": raw[:-64],
        "bad_version": raw[:4] + (7).to_bytes(4, "little") + raw[8:],
    }
    for name, data in cases.items():
        p = str(tmp_path / f"{name}.gguf")
        open(p, "wb").write(data)
        assert not lib.moeb_gguf_open(p.encode()), name
        assert lib.moeb_last_error().decode(), name
    for typ, ne in ((99, (8, 1)), (12, (100, 1))):   # unknown type; 100 values of a 256-value block type
        p = str(tmp_path / f"t{typ}.gguf")
        write_gguf(p, [], [("x", typ, ne, bytes(4096))])
        with pytest.raises(Exception):
            Gguf(p)
    # sizes from the file that would wrap or run past its end: a u8 array of 2^62 elements (its
    # byte count must not seek backwards), a string array longer than the file, and a tensor whose
    # element count overflows 64 bits (its offset + size must not wrap below the file size)
    import struct
    hdr = b"GGUF" + struct.pack("<IQQ", 3, 0, 1)
    arrays = {"huge_u8_array": struct.pack("<IQ", 0, 1 << 62), "huge_str_array": struct.pack("<IQ", 8, 1 << 40)}
    for name, body in arrays.items():
        p = str(tmp_path / f"{name}.gguf")
        open(p, "wb").write(hdr + struct.pack("<Q", 1) + b"a" + struct.pack("<I", 9) + body + bytes(64))
        assert not lib.moeb_gguf_open(p.encode()), name
        assert b"array" in lib.moeb_last_error() or b"truncated" in lib.moeb_last_error(), name
    p = str(tmp_path / "overflow.gguf")
    write_gguf(p, [], [("x", 0, (1 << 31, 1 << 31, 1 << 31, 8), bytes(64))])   # f32: 2^96 x 8 x 4 bytes
    assert not lib.moeb_gguf_open(p.encode())
    assert b"overflow" in lib.moeb_last_error()
    g = Gguf(good)
    assert g.str("gemma4.expert_count") is None          # wrong type asked for
    assert g.u32("general.architecture") is None


def test_loaders_fail_cleanly(tmp_path):
    """Bad arguments, missing pages, pages longer than the slot stride and unreadable files are
    refused before any copy is issued."""
    from llapis_b200 import capi
    from llapis_b200.loader import Store
    lib = capi.lib()
    idx = str(tmp_path / "s.experts.index")
    write_with(lib, idx, idx.replace("index", "pack"), pages())
    st = Store(idx)
    ids = np.array([0, 1], np.int32)            # expert 1 has no page
    dst = C.c_void_p(16)                        # never dereferenced: the page check fails first
    assert lib.moeb_load_store_pages(st.h, 0, 0, 0, ids.ctypes.data, 2, dst, 1 << 20, 0, None) == -1
    assert b"no page" in lib.moeb_last_error()
    ids = np.array([0, 2], np.int32)
    assert lib.moeb_load_store_pages(st.h, 0, 0, 0, ids.ctypes.data, 2, dst, 100, 0, None) == -1   # stride too small
    assert lib.moeb_load_file_range(b"/nonexistent/file", 0, 10, dst, None) == -1
    assert lib.moeb_load_file_range(None, 0, 10, dst, None) == -1
    st.close()
    # a corrupt index: a record count the file cannot hold fails the open (nothing is sized from
    # it), and a page whose offset + size runs past the pack is a bad page, never a huge read
    raw = bytearray(open(idx, "rb").read())
    bad = str(tmp_path / "bad.experts.index")
    import shutil
    shutil.copy(idx.replace("index", "pack"), bad.replace("index", "pack"))
    raw_count = bytearray(raw)
    raw_count[72:80] = (1 << 60).to_bytes(8, "little")                   # record_count
    open(bad, "wb").write(raw_count)
    assert lib.moert_store_verify(bad.encode()) == -1
    assert not lib.moert_store_reader_open(bad.encode(), 0)
    raw_page = bytearray(raw)
    hb = int.from_bytes(raw[12:16], "little")                             # header_bytes
    raw_page[hb + 16:hb + 24] = ((1 << 64) - 8).to_bytes(8, "little")     # record 0: nbytes
    open(bad, "wb").write(raw_page)
    assert lib.moert_store_verify(bad.encode()) == 1
