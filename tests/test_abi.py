"""The C-ABI library loads on a CPU box and exports every symbol the header
declares; argument validation runs host-side (no GPU needed)."""

import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    src = open(os.path.join(ROOT, "include", "mjolnir_b200.h")).read()
    return sorted(set(re.findall(r"^(?:int|const char\*|void|mj_runner\*)\s+(mj_\w+)\(", src, re.M)))


def test_header_symbols_exported():
    from mjolnir_b200 import _lib

    lib = _lib.load()
    declared = _declared()
    assert set(declared) >= {"mj_cache_write", "mj_decode", "mj_combine", "mj_last_error", "mj_create", "mj_plan",
                             "mj_runner_fill", "mj_destroy", "mj_plan_split_kv"}
    for name in declared:
        assert hasattr(lib, name), f"{name} declared in include/mjolnir_b200.h but not exported"
    assert set(_lib.EXPORTED) <= set(declared)
    assert lib.mj_abi_version() == 4
    assert lib.mj_row_bytes(128, _lib.MJ_KV_E2M3) == 96
    assert lib.mj_row_bytes(128, _lib.MJ_KV_FP8_E4M3) == 128
    assert lib.mj_row_bytes(130, _lib.MJ_KV_E2M3) == -1


def test_struct_layouts_match_header():
    """ctypes mirrors of the argument structs have the C sizes (compiled probe)."""
    import subprocess
    import tempfile

    from mjolnir_b200 import _lib

    src = '#include "mjolnir_b200.h"\n#include <stdio.h>\n#include <stddef.h>\nint main(){printf("%zu %zu %zu %zu %zu %zu\\n", sizeof(mj_cache_write_args), sizeof(mj_decode_args), offsetof(mj_decode_args, softmax_scale), offsetof(mj_cache_write_args, status), sizeof(mj_expand_args), offsetof(mj_expand_args, k_ratio));return 0;}\n'
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "probe.c")
        open(c, "w").write(src)
        exe = os.path.join(d, "probe")
        subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), c, "-o", exe], check=True)
        out = subprocess.run([exe], check=True, capture_output=True, text=True).stdout.split()
    sizes = [int(x) for x in out]
    assert sizes[0] == ctypes.sizeof(_lib.CacheWriteArgs)
    assert sizes[1] == ctypes.sizeof(_lib.DecodeArgs)
    assert sizes[2] == _lib.DecodeArgs.softmax_scale.offset
    assert sizes[3] == _lib.CacheWriteArgs.status.offset
    assert sizes[4] == ctypes.sizeof(_lib.ExpandArgs)
    assert sizes[5] == _lib.ExpandArgs.k_ratio.offset


def test_validation_errors_without_gpu():
    """Invalid arguments are rejected on the host with a message, no launch."""
    from mjolnir_b200 import _lib

    a = _lib.DecodeArgs()
    a.num_seqs, a.q_len, a.h_q, a.h_k, a.head_size = 1, 1, 8, 3, 128
    with pytest.raises(_lib.MjolnirError, match="h_q 8 h_k 3"):
        _lib.decode(a, 0)
    a.h_k, a.head_size = 2, 96
    with pytest.raises(_lib.MjolnirError) as e:
        _lib.decode(a, 0)
    assert e.value.code == _lib.MJ_ERR_UNSUPPORTED
    w = _lib.CacheWriteArgs()
    w.num_tokens, w.h_k, w.head_size, w.kv_format = 1, 1, 128, 7
    with pytest.raises(_lib.MjolnirError):
        _lib.cache_write(w, 0)
    x = _lib.ExpandArgs()
    x.num_out_pages, x.h_k, x.page_size, x.num_pages, x.head_size = 1, 1, 16, 1, 120
    with pytest.raises(_lib.MjolnirError, match="head_size 120") as e:
        _lib.expand_pages(x, 0)
    assert e.value.code == _lib.MJ_ERR_UNSUPPORTED


def test_runner_create_fails_cleanly_without_a_gpu_or_bad_shapes():
    """mj_create validates shapes on the host; without a device it returns NULL
    with a message (no crash)."""
    from mjolnir_b200 import _lib

    lib = _lib.load()
    assert not lib.mj_create(0, 8, 3, 128, 16, 4, 1, _lib.MJ_KV_E2M3, 16, 2)  # h_q % h_k
    assert b"invalid" in lib.mj_last_error()
    assert not lib.mj_create(0, 64, 1, 128, 16, 4, 2, _lib.MJ_KV_E2M3, 16, 2)  # 128 rows per KV head
    assert b"64 query rows" in lib.mj_last_error()
