"""The C-ABI library loads and exports every symbol include/*.h declares (CPU only).

No compute call is made here: only version / workspace arithmetic and argument
validation paths that return before any CUDA call.
"""

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def _declared_symbols():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names.update(re.findall(r"\b(tvk_[a-z0-9_]+)\s*\(", text))
    return sorted(names)


@pytest.fixture(scope="module")
def lib():
    from tinyvllm_b200 import build
    build.build()
    from tinyvllm_b200 import _lib
    return _lib.lib()


def test_every_declared_symbol_is_exported(lib):
    names = _declared_symbols()
    assert "tvk_paged_decode_attention" in names
    handle = ctypes.CDLL(str(ROOT / "tinyvllm_b200" / "libtvk.so"))
    missing = [n for n in names if not hasattr(handle, n)]
    assert not missing, f"declared but not exported: {missing}"


def test_python_binding_covers_header(lib):
    from tinyvllm_b200 import _lib
    assert set(_declared_symbols()) <= set(_lib.SIGNATURES), "ctypes prototypes missing for some exports"


def _declared_arity():
    arity = {}
    for h in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        for name, params in re.findall(r"\b(tvk_[a-z0-9_]+)\s*\(([^;{]*?)\)\s*;", text, flags=re.S):
            params = params.strip()
            arity[name] = 0 if params in ("", "void") else params.count(",") + 1
    return arity


def test_binding_argument_counts_match_header():
    from tinyvllm_b200 import _lib
    arity = _declared_arity()
    assert arity, "no declarations parsed"
    for name, n in arity.items():
        assert len(_lib.SIGNATURES[name][1]) == n, f"{name}: header has {n} parameters"


def test_abi_version(lib):
    assert lib.tvk_abi_version() == 1


def test_workspace_size_arithmetic(lib):
    hdr = 256
    # config 1: short tables -> a split size that gives >1 split per sequence
    n = lib.tvk_paged_decode_workspace_size(4, 32, 4, 64, 16, 16, -1)
    assert n > hdr and (n - hdr) % (4 * 32 * (64 + 2) * 4) == 0
    # one split fits -> header only
    assert lib.tvk_paged_decode_workspace_size(4096, 32, 8, 128, 16, 4, -1) == hdr
    # max_context_len truncates the table
    a = lib.tvk_paged_decode_workspace_size(256, 32, 8, 128, 16, 256, -1)
    b = lib.tvk_paged_decode_workspace_size(256, 32, 8, 128, 16, 256, 48)
    assert b == hdr < a


def test_decode_plan(lib):
    plan = (ctypes.c_int * 4)()
    # config 3: 256 sequences x 8 KV heads, 4096-token tables -> persistent CTAs,
    # one 4096-token unit per (sequence, KV head), no combine
    assert lib.tvk_paged_decode_plan(256, 32, 8, 128, 16, 256, -1, 1, plan) == 0
    assert list(plan) == [4096, 1, 1, 1]
    # engine-sized call (64 sequences x 4 KV heads, 64-block tables): one CTA per
    # (sequence, KV head), the whole 1024-token table as one unit, no combine
    assert lib.tvk_paged_decode_plan(64, 32, 4, 64, 16, 64, -1, 1, plan) == 0
    assert list(plan) == [1024, 1, 1, 0]
    # fewer pairs: split to about one wave of CTAs, with a combine
    assert lib.tvk_paged_decode_plan(16, 32, 4, 64, 16, 64, -1, 1, plan) == 0
    assert plan[0] == 256 and plan[1] == 4 and plan[2] == 2 and plan[3] == 0
    # fp32 always takes the one-CTA-per-unit kernel
    assert lib.tvk_paged_decode_plan(256, 32, 8, 128, 16, 256, -1, 0, plan) == 0
    assert plan[3] == 0
    # the workspace covers every plan the sizes can take
    for dt in (0, 1, 2):
        for args in ((256, 32, 8, 128, 16, 256, -1), (64, 32, 4, 64, 16, 64, -1), (4, 32, 4, 64, 16, 16, -1)):
            assert lib.tvk_paged_decode_plan(*args, dt, plan) == 0
            need = 256 + (args[0] * args[1] * plan[1] * (args[3] + 2) * 4 if plan[1] > 1 else 0)
            assert lib.tvk_paged_decode_workspace_size(*args) >= need
    assert lib.tvk_paged_decode_plan(0, 32, 8, 128, 16, 256, -1, 1, plan) == -1


def test_invalid_arguments_are_rejected_before_any_launch(lib):
    rc = lib.tvk_paged_decode_attention(None, None, None, None, None, None, 1, 32, 4, 64, 16, 8, 4, -1, 1,
                                        None, 0, None)
    assert rc == -1 and b"null pointer" in lib.tvk_last_error()
    fake = ctypes.c_void_p(256)
    args = [fake] * 6
    rc = lib.tvk_paged_decode_attention(*args, 1, 30, 4, 64, 16, 8, 4, -1, 1, None, 0, None)
    assert rc == -1 and b"multiple" in lib.tvk_last_error()
    rc = lib.tvk_paged_decode_attention(*args, 1, 32, 4, 96, 16, 8, 4, -1, 1, None, 0, None)
    assert rc == -2
    rc = lib.tvk_paged_decode_attention(*args, 1, 32, 4, 64, 16, 8, 4, -1, 7, None, 0, None)
    assert rc == -1
    # a table wider than one split needs a workspace
    rc = lib.tvk_paged_decode_attention(*args, 1, 32, 4, 64, 16, 8, 64, -1, 1, None, 0, None)
    assert rc == -4 and b"workspace" in lib.tvk_last_error()
    assert lib.tvk_paged_decode_attention(*args, 0, 32, 4, 64, 16, 8, 4, -1, 1, None, 0, None) == 0


def test_cpu_tensors_are_refused():
    import torch
    from tinyvllm_b200.attention import paged_decode_attention
    q = torch.zeros(1, 1, 4, 32)
    kc = torch.zeros(2, 16, 4, 32)
    with pytest.raises(RuntimeError, match="CUDA"):
        paged_decode_attention(q, kc, kc, torch.zeros(1, 2, dtype=torch.int32),
                               torch.ones(1, dtype=torch.int32), 4, 4, 32, 16)


def test_wait_test_hook_rejects_limits_out_of_range(lib):
    assert lib.tvk_debug_arm_wait_timeout(10) == -1
    assert lib.tvk_debug_arm_wait_timeout(3_000_000_000) == -1
    assert b"wait limit" in lib.tvk_last_error()


def test_noalloc_status_rejects_null(lib):
    assert lib.tvk_paged_decode_noalloc_status(None, None) == -1


def test_probes_reject_bad_arguments(lib):
    # argument checks run before any CUDA call
    assert lib.tvk_probe_mma_issue(96, 16, None, 1, None) != 0
    assert lib.tvk_probe_mma_issue(128, 16, None, 1, None) != 0
    assert lib.tvk_probe_exp_unit(7, 16, None, 1, None, None) != 0
    assert lib.tvk_probe_exp_unit(0, 0, None, 1, None, None) != 0
