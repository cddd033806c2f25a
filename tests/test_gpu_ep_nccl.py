"""The expert-parallel layer on 2 GPUs over NCCL (zunzuncito_b200/ep.py with the device
pack/unpack kernels and zz_moe_ffn_q8_dev): each rank holds half of the experts and its
own tokens, and its output must equal the single-GPU batch-union layer over the full bank
(itself checked against the oracle in test_gpu_moe.py). Skipped on boxes with fewer than
2 GPUs."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch

from zunzuncito_b200 import synth

pytestmark = pytest.mark.gpu

E, D, MI, K, S = 8, 256, 128, 4, 96


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _bank_blobs():
    import oracle
    orc = oracle.Oracle()
    return np.stack([np.concatenate([orc.q40_quant_rows(synth.gaussian(900 + 3 * e + i, shp, 0.02)).ravel()
                                     for i, shp in enumerate([(MI, D), (MI, D), (D, MI)])]) for e in range(E)])


def _worker(rank, world, port, out_dir):
    import torch.distributed as dist
    import zunzuncito_b200 as zz
    from zunzuncito_b200.ep import ep_moe_layer
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    try:
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
        per = E // world
        blobs = torch.from_numpy(_bank_blobs()[rank * per:(rank + 1) * per]).cuda()
        bank = zz.ExpertBankDev(zz.GPU_FMT_Q40, blobs, D, MI)
        X = torch.from_numpy(synth.gaussian(950 + rank, (S, D))).cuda()
        e, w, _ = synth.zipf_routing(960 + rank, S, E, K)
        eidx, ewt = torch.from_numpy(e).cuda(), torch.from_numpy(w).cuda()
        xq, xs, _ = zz.quant_act(X)
        ffn = lambda q, s, ee, ww: zz.moe_ffn_q8(bank, q, s, ee, ww, zz.ZZ_ACT_GEGLU_TANH)
        out = ep_moe_layer(xq, xs, eidx, ewt, E, ffn)
        np.save(os.path.join(out_dir, f"out{rank}.npy"), out.cpu().numpy())
        dist.barrier()
    except Exception as ex:  # noqa: BLE001
        with open(os.path.join(out_dir, f"err{rank}.txt"), "w") as f:
            f.write(repr(ex))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep_two_gpus_match_single_gpu(tmp_path):
    import torch.multiprocessing as mp
    import zunzuncito_b200 as zz
    mp.start_processes(_worker, args=(2, _port(), str(tmp_path)), nprocs=2, start_method="spawn")
    bank = zz.ExpertBankDev(zz.GPU_FMT_Q40, torch.from_numpy(_bank_blobs()).cuda(), D, MI)
    for r in range(2):
        assert not (tmp_path / f"err{r}.txt").exists(), (tmp_path / f"err{r}.txt").read_text()
        X = torch.from_numpy(synth.gaussian(950 + r, (S, D))).cuda()
        e, w, _ = synth.zipf_routing(960 + r, S, E, K)
        want = zz.moe_ffn(bank, X, torch.from_numpy(e).cuda(), torch.from_numpy(w).cuda(),
                          zz.ZZ_ACT_GEGLU_TANH).cpu().numpy()
        got = np.load(tmp_path / f"out{r}.npy")
        assert np.max(np.abs(got - want)) <= 1e-5 * np.max(np.abs(want)), r
