"""Expert-parallel exchange logic (zunzuncito_b200/ep.py) on CPU ranks over gloo: two
ranks, each holding half of the experts and its own tokens, must reproduce the
single-process batch-union layer of the oracle on the union of their tokens. A second
case shows a rank failure surfacing on the host as an error, not a hang."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from zunzuncito_b200 import synth

E, D, MI, K, S = 8, 128, 64, 2, 6


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _blobs(orc, kind):
    if kind == 3:
        return np.stack([np.concatenate([synth.tq2_tensor(50 + 3 * e + i, o, i_) for i, (o, i_) in
                                         enumerate([(MI, D), (MI, D), (D, MI)])]) for e in range(E)])
    return np.stack([np.concatenate([orc.q40_quant_rows(synth.gaussian(50 + 3 * e + i, shp, 0.02)).ravel()
                                     for i, shp in enumerate([(MI, D), (MI, D), (D, MI)])]) for e in range(E)])


def _worker(rank, world, port, kind, out_dir, fail_rank):
    import oracle
    from zunzuncito_b200.ep import ep_moe_layer
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    orc = oracle.Oracle()
    blobs = _blobs(orc, kind)
    per = E // world
    mine = blobs[rank * per:(rank + 1) * per]
    X = synth.gaussian(70 + rank, (S, D))
    eidx, ewt, _ = synth.zipf_routing(80 + rank, S, E, K)
    xq, xs = orc.quant_act(X)

    def ffn(q, s, e, w):
        o = orc.moe_layer_q8(kind, mine, q.numpy(), s.numpy(), e.numpy(), w.numpy(), D, MI, 7.0)
        return torch.from_numpy(o)

    try:
        if rank == fail_rank:
            raise RuntimeError("injected failure before the dispatch")
        out = ep_moe_layer(torch.from_numpy(xq), torch.from_numpy(xs), torch.from_numpy(eidx),
                           torch.from_numpy(ewt), E, ffn)
        np.save(os.path.join(out_dir, f"out{rank}.npy"), out.numpy())
    except Exception as e:  # noqa: BLE001
        with open(os.path.join(out_dir, f"err{rank}.txt"), "w") as f:
            f.write(repr(e))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


@pytest.mark.parametrize("kind", [0, 3])
def test_ep_two_ranks_match_single_process(orc, tmp_path, kind):
    mp.start_processes(_worker, args=(2, _port(), kind, str(tmp_path), -1), nprocs=2, start_method="fork")
    blobs = _blobs(orc, kind)
    for r in range(2):
        assert not (tmp_path / f"err{r}.txt").exists(), (tmp_path / f"err{r}.txt").read_text()
        X = synth.gaussian(70 + r, (S, D))
        eidx, ewt, _ = synth.zipf_routing(80 + r, S, E, K)
        want = orc.moe_layer(kind, blobs, X, eidx, ewt, D, MI, 7.0)
        got = np.load(tmp_path / f"out{r}.npy")
        assert np.max(np.abs(got - want)) <= 1e-5 * np.max(np.abs(want))


def test_ep_rank_failure_is_reported(tmp_path):
    """rank 1 dies before the exchange; rank 0's collective must end with an error
    (process-group timeout or peer loss) instead of waiting forever."""
    mp.start_processes(_worker, args=(2, _port(), 0, str(tmp_path), 1), nprocs=2, start_method="fork", join=True)
    assert (tmp_path / "err1.txt").exists()
    assert (tmp_path / "err0.txt").exists()
    assert not (tmp_path / "out0.npy").exists()


def _uneven_worker(rank, world, port, out_dir):
    from zunzuncito_b200.ep import ep_moe_layer
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    try:
        xq = torch.zeros((S, D), dtype=torch.int8)
        xs = torch.zeros((S, D // 32))
        eidx = torch.zeros((S, K), dtype=torch.int32)
        ewt = torch.zeros((S, K))
        ep_moe_layer(xq, xs, eidx, ewt, 7, lambda *a: None)   # 7 experts over 2 ranks
    except ValueError as e:
        with open(os.path.join(out_dir, f"val{rank}.txt"), "w") as f:
            f.write(str(e))
    finally:
        dist.destroy_process_group()


def test_ep_rejects_uneven_expert_split(tmp_path):
    """experts that do not divide over the ranks would leave the remainder on no rank
    (their contributions silently dropped); the layer refuses before any exchange"""
    mp.start_processes(_uneven_worker, args=(2, _port(), str(tmp_path)), nprocs=2, start_method="fork")
    for r in range(2):
        assert "shard evenly" in (tmp_path / f"val{r}.txt").read_text()
