"""CPU checks of the C ABI: the in-tree library loads without a GPU and
exports every entry point the headers under include/ declare."""
import ctypes
import pathlib
import re

from conftest import ROOT, load_pkg

HEADERS = sorted((ROOT / "include").glob("*.h"))


def declared_functions():
    names = set()
    for h in HEADERS:
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names |= set(re.findall(r"\b(?:int|int64_t)\s+(b2_\w+)\s*\(", text))
    return sorted(names)


def test_header_declares_entry_points():
    names = declared_functions()
    assert {"b2_append_rope", "b2_decode_attn", "b2_combine", "b2_last_error", "b2_version",
            "b2_exchange_bytes", "b2_add_rmsnorm", "b2_swiglu", "b2_shortconv_step", "b2_argmax_rows"} <= set(names)


def test_block_entry_points_check_arguments_without_gpu():
    lib = load_pkg("_lib")
    cdll = lib.load()
    assert cdll.b2_add_rmsnorm(None, None, None, ctypes.c_float(1e-5), None, None, 1, 1024, None) == lib.B2_ERR_ARG
    assert "null pointer" in lib.last_error()
    assert cdll.b2_swiglu(None, None, 0, 2560, None) == lib.B2_OK      # no rows: nothing to do
    assert cdll.b2_shortconv_step(None, None, None, None, 2, 1024, None) == lib.B2_ERR_ARG


def test_library_exports_every_declared_symbol():
    lib = load_pkg("_lib")
    cdll = lib.load()
    for name in declared_functions():
        assert hasattr(cdll, name), name
        assert name in lib.SIGNATURES, f"{name} has no ctypes signature"


def test_version_and_error_text_without_gpu():
    lib = load_pkg("_lib")
    assert lib.load().b2_version() >= 100
    # argument checks run on the host before any CUDA call
    rc = lib.load().b2_decode_attn(None, None, None, 1, None, 1, None, 1, 1, 1,
                                   ctypes.c_float(0.125), None, None, None, None)
    assert rc == lib.B2_ERR_ARG
    assert "null pointer" in lib.last_error()
    rc = lib.load().b2_append_rope(None, 2048, None, None, ctypes.c_float(1e-5), None, None, 0, None,
                                   None, 0, None, None, 0, None, 0, 7, None, None)
    assert rc == lib.B2_OK   # batch 0 is a no-op


def test_library_lives_in_tree():
    lib = load_pkg("_lib")
    assert pathlib.Path(lib.LIB_PATH).parent.name == "ryzenai-npu-lab_b200"


def test_decode_step_exchange_argument_checks_without_gpu():
    """The torch wrapper refuses an exchange without an output or with states
    (host checks before any launch), and the C entry rejects a bad world."""
    import torch
    attn = load_pkg("attention")
    lib = load_pkg("_lib")
    bf, i32 = torch.bfloat16, torch.int32
    qkv = torch.zeros(1, 2048, dtype=bf)
    past = torch.zeros(1, dtype=i32)
    pool = torch.zeros(2, 8, 64, 64, dtype=bf)
    tables = torch.zeros(1, 2, dtype=i32)
    part_ml = torch.zeros(1, 2, 16, 2)
    part_o = torch.zeros(1, 2, 16, 64)
    counters = torch.zeros(10, dtype=i32)
    err = torch.zeros(1, dtype=i32)
    kw = dict(k_pool=pool, v_pool=pool, block_tables=tables, blocks_per_split=1, part_ml=part_ml, part_o=part_o,
              counters=counters, dev_err=err, mode=lib.B2_STORE_KV, exchange=(None, 2, 0))
    import pytest
    with pytest.raises(ValueError, match="exchange"):
        attn.decode_step(qkv, past, out=None, **kw)
    with pytest.raises(ValueError, match="exchange"):
        attn.decode_step(qkv, past, out=torch.zeros(1, 16, 64, dtype=bf), state_ml=torch.zeros(1, 16, 2),
                         state_o=torch.zeros(1, 16, 64), **kw)
    rc = lib.load().b2_decode_step_exchange(None, 2048, None, None, ctypes.c_float(1e-5), None, None, 0, None, None,
                                            None, 1, None, None, 1, 1, 1, ctypes.c_float(0.125), 0, None, None,
                                            None, None, None, 0, None, 9, 0, None, None)
    assert rc == lib.B2_ERR_ARG and "world" in lib.last_error()


def test_argument_errors_without_gpu():
    """Host-side refusals (B2_ERR_ARG with a message, before any CUDA call)."""
    lib = load_pkg("_lib")
    c = lib.load()
    f = ctypes.c_float
    buf = ctypes.create_string_buffer(64)

    def refused(rc, text):
        assert rc == lib.B2_ERR_ARG, rc
        assert text in lib.last_error(), lib.last_error()

    # decode step: more than 64 blocks per split
    refused(c.b2_decode_step(buf, 2048, None, None, f(1e-5), None, None, 0, buf, None, buf, 70, buf, buf, 10,
                             1, 65, f(0.125), 0, buf, None, None, None, buf, buf, buf, 0, buf, None),
            "blocks_per_split")
    # block tables wider than an int32 token count can address (2^25 blocks of 64 tokens)
    wide = 1 << 25
    refused(c.b2_decode_step(buf, 2048, None, None, f(1e-5), None, None, 0, buf, None, buf, wide, buf, buf, 10,
                             1, 1, f(0.125), 0, buf, None, None, None, buf, buf, buf, 0, buf, None),
            "max_blocks_per_seq")
    refused(c.b2_decode_attn(buf, buf, buf, 10, buf, wide, buf, 1, 1, wide, f(0.125), buf, buf, buf, None),
            "max_blocks_per_seq")
    refused(c.b2_decode_attn(buf, buf, buf, 10, buf, 4, buf, 1, wide, 1, f(0.125), buf, buf, buf, None),
            "blocks_per_split")
    refused(c.b2_prefill_attn(buf, buf, buf, 10, buf, wide, buf, None, 4, 1, f(0.125), buf, buf, None),
            "max_blocks_per_seq")
    refused(c.b2_append_rope(buf, 2048, None, None, f(1e-5), None, None, 0, buf, buf, wide, buf, buf, 10, None,
                             1, 4, buf, None), "max_blocks_per_seq")
    refused(c.b2_combine(buf, buf, 1 << 20, buf, 64, 1, buf, None, None, None), "int32 token count")
    # prefill split: batch x splits beyond the grid limit
    refused(c.b2_prefill_attn_split(buf, buf, buf, 10, buf, 100000, buf, None, 4, 2, f(0.125), 1, buf, buf, buf,
                                    buf, None), "65535")
    # exchange: world beyond the maximum, rank outside the world
    areas = (ctypes.c_void_p * 2)(ctypes.addressof(buf), ctypes.addressof(buf))
    refused(c.b2_exchange_merge(buf, buf, 1, areas, 9, 0, buf, buf, None), "world")
    refused(c.b2_exchange_merge(buf, buf, 1, areas, 2, 2, buf, buf, None), "rank")
    # layer kernels: width not a multiple of 8, odd SwiGLU width
    refused(c.b2_add_rmsnorm(buf, None, buf, f(1e-5), None, buf, 1, 1020, None), "width")
    refused(c.b2_swiglu(buf, buf, 1, 7, None), "ffn")
    refused(c.b2_argmax_rows(buf, 1, 12, None, None), "null pointer")
    # host-fed pipeline: slot outside 0 / 1
    refused(c.b2_decode_step_host2(buf, buf, buf, buf, buf, buf, 2, None, None, f(1e-5), None, None, 0, buf, 1,
                                   buf, buf, 1, 1, 1, f(0.125), buf, buf, buf, buf, None), "slot")


def test_rope_tables_must_be_64_wide_without_gpu():
    """Every wrapper that rotates q/k refuses cos/sin tables that are not
    [positions, 64] before any launch (the kernels index rows of 64)."""
    import pytest
    import torch
    attn = load_pkg("attention")
    lib = load_pkg("_lib")
    bf, i32 = torch.bfloat16, torch.int32
    past = torch.zeros(1, dtype=i32)
    pool = torch.zeros(2, 8, 64, 64, dtype=bf)
    tables = torch.zeros(1, 2, dtype=i32)
    err = torch.zeros(1, dtype=i32)
    mode = lib.B2_ROPE_QK | lib.B2_STORE_KV
    for cos in (torch.zeros(16, 32, dtype=bf), torch.zeros(1024, dtype=bf), torch.zeros(0, 64, dtype=bf)):
        sin = cos.clone()
        with pytest.raises(ValueError, match="cos/sin"):
            attn.append_rope(torch.zeros(1, 2048, dtype=bf), past, q_out=None, dev_err=err, mode=mode, cos=cos,
                             sin=sin, k_pool=pool, v_pool=pool, block_tables=tables)
        with pytest.raises(ValueError, match="cos/sin"):
            attn.decode_step(torch.zeros(1, 2048, dtype=bf), past, k_pool=pool, v_pool=pool, block_tables=tables,
                             blocks_per_split=1, out=torch.zeros(1, 16, 64, dtype=bf),
                             part_ml=torch.zeros(1, 2, 16, 2), part_o=torch.zeros(1, 2, 16, 64),
                             counters=torch.zeros(10, dtype=i32), dev_err=err, mode=mode, cos=cos, sin=sin)
        with pytest.raises(ValueError, match="cos/sin"):
            attn.prefill(torch.zeros(1, 4, 2048, dtype=bf), past, k_pool=pool, v_pool=pool, block_tables=tables,
                         gamma_q=None, gamma_k=None, cos=cos, sin=sin, dev_err=err, mode=mode)


def test_reference_binding_matches_the_library_signatures():
    """The standalone ctypes stub a maintainer adds to the reference's loop
    (reference_binding.py) declares the same argument types as _lib.py, and
    binds the loaded library without a GPU."""
    lib = load_pkg("_lib")
    rb = load_pkg("reference_binding")
    assert {"b2_append_rope", "b2_decode_attn", "b2_combine", "b2_decode_step"} <= set(rb.ARGTYPES)
    for name, args in rb.ARGTYPES.items():
        assert list(args) == list(lib.SIGNATURES[name][1]), name
    cdll = rb.bind(str(lib.LIB_PATH))
    assert cdll.b2_decode_step_counters(4) == 2 + 8 * 4
    assert cdll.b2_combine(None, None, 0, None, 1, 1, None, None, None, None) == lib.B2_ERR_ARG
    assert "num_parts" in rb.last_error(cdll)


def test_wait_limits_without_gpu():
    """b2_set_wait_limits: defaults 2 s / 5 s, <= 0 restores them, > 60 s refused."""
    lib = load_pkg("_lib")
    c = lib.load()
    w, q = ctypes.c_int64(), ctypes.c_int64()
    assert c.b2_get_wait_limits(ctypes.byref(w), ctypes.byref(q)) == lib.B2_OK
    assert (w.value, q.value) == (2_000_000_000, 5_000_000_000)
    assert c.b2_set_wait_limits(1_000_000, 3_000_000) == lib.B2_OK
    c.b2_get_wait_limits(ctypes.byref(w), ctypes.byref(q))
    assert (w.value, q.value) == (1_000_000, 3_000_000)
    assert c.b2_set_wait_limits(61_000_000_000, 0) == lib.B2_ERR_ARG
    assert "60" in lib.last_error()
    assert c.b2_set_wait_limits(0, -1) == lib.B2_OK
    c.b2_get_wait_limits(ctypes.byref(w), ctypes.byref(q))
    assert (w.value, q.value) == (2_000_000_000, 5_000_000_000)


def test_noalloc_refuses_token_count_overflow_without_gpu():
    """b2_decode_attn_noalloc refuses a split geometry whose token count
    (splits x blocks_per_split x 64) leaves int32, before any launch."""
    lib = load_pkg("_lib")
    c = lib.load()
    buf = ctypes.create_string_buffer(64)
    big = (1 << 25) - 1
    rc = c.b2_decode_attn_noalloc(buf, buf, buf, 1, buf, big, buf, 1, big // 2 + 1, ctypes.c_float(0.125),
                                  buf, buf, None)
    assert rc == lib.B2_ERR_ARG
    assert "int32" in lib.last_error()


def test_last_error_is_per_thread_without_gpu():
    """b2_last_error reports the calling thread's own last error: two threads
    fail different calls in turn, then each reads its own message."""
    import threading
    lib = load_pkg("_lib")
    c = lib.load()
    buf = ctypes.create_string_buffer(64)
    gate = threading.Barrier(2)
    seen = {}

    def worker(name, call, expect):
        def text():
            out = ctypes.create_string_buffer(512)
            c.b2_last_error(out, 512)
            return out.value.decode()
        if name == "a":
            call()
            gate.wait()      # a has failed
            gate.wait()      # b has failed too
        else:
            gate.wait()
            call()
            gate.wait()
        seen[name] = (expect in text(), text())

    calls = {
        "a": (lambda: c.b2_swiglu(buf, buf, 1, 7, None), "ffn"),
        "b": (lambda: c.b2_argmax_rows(buf, 1, 12, None, None), "null pointer"),
    }
    threads = [threading.Thread(target=worker, args=(n, *calls[n])) for n in calls]
    for t in threads:
        t.start()
    for t in threads:
        t.join(30)
    assert seen["a"][0] and "ffn" in seen["a"][1] and "null pointer" not in seen["a"][1], seen
    assert seen["b"][0] and "ffn" not in seen["b"][1], seen


def test_stall_bit_is_refused_outside_the_decode_step_without_gpu():
    """B2_TEST_STALL (a test of the failure path) belongs to b2_decode_step
    only: the append entry points refuse it before any launch."""
    lib = load_pkg("_lib")
    c = lib.load()
    buf = ctypes.create_string_buffer(64 * 1024)
    rc = c.b2_append_rope(buf, 2048, None, None, ctypes.c_float(1e-5), None, None, 0, buf, None, 0, None, None, 0,
                          None, 1, lib.B2_TEST_STALL, buf, None)
    assert rc == lib.B2_ERR_ARG and "mode" in lib.last_error()
    rc = c.b2_prefill_append(buf, 2048, None, None, ctypes.c_float(1e-5), None, None, 0, buf, None, 1, None, 0,
                             None, None, 0, None, 1, lib.B2_TEST_STALL, buf, None)
    assert rc == lib.B2_ERR_ARG and "mode" in lib.last_error()
