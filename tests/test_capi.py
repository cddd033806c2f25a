"""The C-ABI library without a GPU: it loads, exports every entry point that
include/zz_gpu.h declares, and declines cleanly (0 + a reason) when there is no device."""
import ctypes
import os
import re

import pytest
import torch

import zunzuncito_b200 as zz

HDR = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "zz_gpu.h")


def declared_symbols():
    txt = open(HDR).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b((?:gpu|zz)_\w+)\s*\(", txt)))


def test_header_symbols_exported():
    lib = ctypes.CDLL(zz.LIB_PATH)
    syms = declared_symbols()
    assert len(syms) >= 20
    missing = [s for s in syms if not hasattr(lib, s)]
    assert not missing, missing


def test_python_prototypes_cover_header():
    names = {p[0] for p in zz._PROTOS}
    assert set(declared_symbols()) <= names


def test_library_is_sm100a():
    data = open(zz.LIB_PATH, "rb").read()
    assert b"sm_100a" in data


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-device decline")
def test_declines_without_device():
    assert zz.lib.gpu_init() == 0
    assert zz.lib.gpu_ready() == 0
    assert len(zz.lib.gpu_last_error()) > 0
    y = (ctypes.c_float * 4)()
    assert zz.lib.gpu_matmul(1, y, None, None, 4, 32, 1) == 0
    assert zz.lib.gpu_name() == b"none"


def test_size_queries_host_only():
    assert zz.lib.zz_qtensor_bytes(zz.GPU_FMT_Q40, 2816, 2816) >= 2816 * 1408 + 2816 * 88 * 2
    assert zz.lib.zz_qtensor_bytes(zz.GPU_FMT_TQ2, 10, 96) == 0   # tq2 needs I % 64
    assert zz.lib.zz_qtensor_bytes(zz.GPU_FMT_Q4A, 10, 64) == 512 + 256  # q4a planes, each 256-aligned
    assert zz.lib.zz_qtensor_bytes(zz.GPU_FMT_Q4A, 10, 96) == 0   # q4a needs I % 64
    assert zz.lib.zz_expert_bank_bytes(zz.GPU_FMT_Q40, 128, 2816, 704) > 128 * 3345408 * 0.99
    assert zz.lib.zz_expert_bank_bytes(zz.GPU_FMT_Q40, 128, 2816, 700) == 0  # inter % 64
    b = zz.ExpertBank(zz.GPU_FMT_Q40, 128, 2816, 704, None, None, None, None)
    assert zz.lib.zz_moe_workspace_bytes(ctypes.byref(b), 512, 8) > 512 * 8 * 704


def test_bad_arguments_decline_before_device_work():
    t = zz.QTensor(zz.GPU_FMT_Q40, 16, 33, None, None)
    assert zz.lib.zz_matvec_dev(ctypes.byref(t), None, None, None, None, 1, None) == 0
    assert b"invalid" in zz.lib.gpu_last_error()
    assert zz.lib.zz_quant_act_dev(None, 1, 48, None, None, None, None) == 0


def test_ep_exchange_entries_host_checks():
    """the expert-parallel row layout size, and argument checks that decline before any
    device work"""
    assert zz.lib.zz_ep_row_bytes(2816, 8) == 2816 + 88 * 4 + 8 * 8   # 3232
    assert zz.lib.zz_ep_row_bytes(2048, 8) == 2048 + 64 * 4 + 64
    p = ctypes.c_void_p(16)
    assert zz.lib.zz_ep_pack_dev(p, p, p, p, 4, 33, 8, 2, 64, p, None) == 0          # D % 32
    assert b"bad shape" in zz.lib.gpu_last_error()
    assert zz.lib.zz_ep_pack_dev(p, p, p, p, 4, 64, 8, 0, 64, p, None) == 0          # world 0
    assert zz.lib.zz_ep_pack_dev(None, p, p, p, 4, 64, 8, 2, 64, p, None) == 0       # null
    assert b"null" in zz.lib.gpu_last_error()
    assert zz.lib.zz_ep_pack_dev(ctypes.c_void_p(18), p, p, p, 4, 64, 8, 2, 64, p, None) == 0  # alignment
    assert zz.lib.zz_ep_pack_dev(None, None, None, None, 0, 64, 8, 2, 64, None, None) == 1   # S = 0: nothing
    assert zz.lib.zz_ep_unpack_dev(p, 3, 64, 0, p, p, p, p, None) == 0                # K <= 0
    assert zz.lib.zz_ep_unpack_dev(p, 0, 64, 8, p, p, p, p, None) == 1                # R = 0: nothing


def test_lazy_load_names_match_api():
    """the package resolves exactly api.__all__ lazily, and importing the package or its
    CPU-side modules maps no CUDA library (the benchmark's reference arm relies on it)"""
    import subprocess
    import sys
    from zunzuncito_b200 import api
    assert set(api.__all__) == set(zz._API_NAMES)
    code = ("import zunzuncito_b200, zunzuncito_b200.synth, zunzuncito_b200.ep; "
            "print('libzz_cuda' in open('/proc/self/maps').read())")
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, check=True,
                         cwd=os.path.dirname(os.path.dirname(HDR)))
    assert out.stdout.strip() == "False"


@pytest.mark.parametrize("fmt,E,D,MI,smax", [(zz.GPU_FMT_Q40, 128, 2816, 704, 862), (zz.GPU_FMT_TQ2, 256, 2048, 512, 1147)])
def test_noalloc_capacity_matches_header(fmt, E, D, MI, smax):
    """the largest S the allocation-free entry point takes at top-8, as its header states:
    the workspace of S fits the fixed scratch array, that of S + 1 does not"""
    cap = int(re.search(r"#define ZZ_NOALLOC_SCRATCH_BYTES \((\d+)u << (\d+)\)", open(HDR).read()).group(1)) << 20
    assert cap == 32 << 20
    b = zz.ExpertBank(fmt, E, D, MI, None, None, None, None)
    assert zz.lib.zz_moe_workspace_bytes(ctypes.byref(b), smax, 8) <= cap
    assert zz.lib.zz_moe_workspace_bytes(ctypes.byref(b), smax + 1, 8) > cap
    assert f"S > {smax}" in open(HDR).read()


def test_workspace_follows_engine(monkeypatch):
    """the layer's workspace holds the fp16 operand planes of the tcgen05 engines only for
    calls those engines take: the hidden rows' planes (4 bytes per element) from the
    prefill size on (experts averaging >= 128 routed rows: S = 2048 at top-8 over 128
    experts), the gathered activation rows' planes too when h3 is forced"""
    monkeypatch.delenv("ZZ_MOE_KERNEL", raising=False)
    b = zz.ExpertBank(zz.GPU_FMT_Q40, 128, 2816, 704, None, None, None, None)
    ws = lambda S: zz.lib.zz_moe_workspace_bytes(ctypes.byref(b), S, 8)  # noqa: E731
    step = ws(2047) - ws(2046)
    assert ws(2048) - ws(2047) > 2047 * 8 * 704 * 4          # the hidden planes appear
    monkeypatch.setenv("ZZ_MOE_KERNEL", "mma8w")
    assert ws(2048) - ws(2047) < 4 * step                    # no planes on mma.sync alone
    monkeypatch.setenv("ZZ_MOE_KERNEL", "mma8")
    plain = ws(512)
    monkeypatch.setenv("ZZ_MOE_KERNEL", "h3")
    assert ws(512) - plain >= 512 * 8 * (2816 + 704) * 4    # both operand planes
    q8 = zz.ExpertBank(zz.GPU_FMT_Q80, 128, 2816, 704, None, None, None, None)
    monkeypatch.delenv("ZZ_MOE_KERNEL")
    w8 = lambda S: zz.lib.zz_moe_workspace_bytes(ctypes.byref(q8), S, 8)  # noqa: E731
    assert w8(2048) - w8(2047) < 4 * (w8(2047) - w8(2046))   # q8_0 banks stay on mma.sync
