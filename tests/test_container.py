"""The gemma4 container loader (zz_container_*): the manifest parser against the
reference's own manifest() on the same files (no GPU), and on the GPU the loaded expert
bank / dense planes against ones packed from the same bytes directly."""
import ctypes
import os

import numpy as np
import pytest

import zunzuncito_b200 as zz
from tests import container_fixture


@pytest.fixture(scope="module")
def container(orc, tmp_path_factory):
    d = str(tmp_path_factory.mktemp("g4c"))
    info = container_fixture.write(d, orc)
    return d, info


def _open(d):
    h = ctypes.c_void_p()
    assert zz.lib.zz_container_open(d.encode(), ctypes.byref(h)) == 1, zz.lib.gpu_last_error()
    return h


def test_manifest_parse(container):
    d, info = container
    h = _open(d)
    try:
        v = ctypes.c_double()
        assert zz.lib.zz_container_cfg(h, b"hidden", ctypes.byref(v)) == 1 and v.value == 256
        assert zz.lib.zz_container_cfg(h, b"final_logit_softcap", ctypes.byref(v)) == 1 and v.value == 30.0
        assert zz.lib.zz_container_cfg(h, b"nope", ctypes.byref(v)) == 0
        fmt, O, I = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        off, ln = ctypes.c_int64(), ctypes.c_int64()
        assert zz.lib.zz_container_dense_info(h, b"embed_tokens", ctypes.byref(fmt), ctypes.byref(O), ctypes.byref(I),
                                              ctypes.byref(off), ctypes.byref(ln)) == 1
        assert (fmt.value, O.value, I.value, off.value, ln.value) == (1, 512, 256, 0, info["embed"].size)
        for (li, e), o in info["offsets"].items():
            assert zz.lib.zz_container_expert_offset(h, li, e) == o
        assert zz.lib.zz_container_expert_offset(h, 2, 0) == -1
        assert zz.lib.zz_container_bank_bytes(h) == zz.lib.zz_expert_bank_bytes(zz.GPU_FMT_Q40, 8, 256, 128)
    finally:
        zz.lib.zz_container_close(h)


def test_manifest_matches_reference_parser(container, ref):
    """the reference engine's manifest() (gemma4.c:260-403) on the same directory reads
    the same expert offsets and blob geometry"""
    d, info = container
    esz3 = (ctypes.c_longlong * 3)()
    eoff = (ctypes.c_longlong * 16)()
    f = ref.fn("gemma4_manifest", ctypes.c_int, [ctypes.c_char_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int])
    assert f(d.encode(), esz3, eoff, 16) == 16
    assert tuple(esz3) == info["esz"]
    h = _open(d)
    try:
        for i in range(16):
            assert zz.lib.zz_container_expert_offset(h, i // 8, i % 8) == eoff[i]
    finally:
        zz.lib.zz_container_close(h)


def test_open_missing_dir(tmp_path):
    h = ctypes.c_void_p()
    assert zz.lib.zz_container_open(str(tmp_path / "none").encode(), ctypes.byref(h)) == 0
    assert b"manifest.txt" in zz.lib.gpu_last_error()


@pytest.mark.gpu
def test_load_bank_and_dense(container, orc):
    import torch
    from zunzuncito_b200 import synth
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    d, info = container
    h = _open(d)
    try:
        mem = zz.alloc_aligned(zz.lib.zz_container_bank_bytes(h))
        bank = zz.ExpertBank()
        st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        assert zz.lib.zz_container_load_bank_dev(h, 1, ctypes.c_void_p(mem.data_ptr()), ctypes.byref(bank), st) == 1, \
            zz.lib.gpu_last_error()
        direct = zz.ExpertBankDev(zz.GPU_FMT_Q40, torch.from_numpy(np.stack(info["blobs"][1])).cuda(), 256, 128)
        assert torch.equal(mem, direct.mem)   # the same planes, byte for byte
        tq = zz.QTensor()
        tm = zz.alloc_aligned(zz.lib.zz_qtensor_bytes(zz.GPU_FMT_Q40, 512, 256))
        assert zz.lib.zz_container_load_dense_dev(h, b"embed_tokens", ctypes.c_void_p(tm.data_ptr()), ctypes.byref(tq),
                                                  st) == 1, zz.lib.gpu_last_error()
        x = synth.gaussian(5, (1, 256))
        xq, sx = orc.quant_act(x)
        xq_d, sx_d = torch.from_numpy(xq).cuda(), torch.from_numpy(sx).cuda()
        y = torch.empty(512, device="cuda")
        assert zz.lib.zz_lm_head_dev(ctypes.byref(tq), ctypes.c_void_p(xq_d.data_ptr()), ctypes.c_void_p(sx_d.data_ptr()),
                                     None, 30.0, ctypes.c_void_p(y.data_ptr()), st) == 1
        want = np.tanh(orc.q40_matvec(info["embed"].reshape(512, -1), xq[0], sx[0]).astype(np.float64) / 30) * 30
        assert np.max(np.abs(y.cpu().numpy() - want)) <= 1e-4 * np.max(np.abs(want))
    finally:
        zz.lib.zz_container_close(h)
