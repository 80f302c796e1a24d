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
