"""Tensor parallelism on 2 GPUs (one process per GPU, NCCL through the
library's own communicator): a block-format model split over 2 ranks gives
the logits of the unsharded oracle within tolerance and the same 64 greedy
tokens, unless the oracle's top-2 margin at the first divergence is below
the observed logit error.
Skipped on boxes with fewer than 2 GPUs."""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
STEPS = 64
PROMPT = [7, 8, 9, 100, 200, 11, 12, 13]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _weights(fmt, name):
    from synapse_b200 import synth
    from oracle import oracle as O
    cfg = synth.lm_config(name)
    w = synth.gen_lm_weights(cfg, fmt, seed=31,
                             dequant=lambda f, b, n: O.dequant(f.name, b, n)[1])
    return cfg, w


def _rank(rank, world, port, fmt, name, q, peer="0"):
    import sys
    sys.path.insert(0, ROOT)
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port),
                      SYN_TP_PEER_ALLREDUCE=peer)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        _run_rank(rank, world, fmt, name, q, dist)
    except Exception as e:  # report instead of leaving the parent waiting
        q.put(("error", rank, repr(e)))
        raise
    finally:
        dist.destroy_process_group()


def _run_rank(rank, world, fmt, name, q, dist):
    if True:
        import synapse_b200 as sb
        torch.cuda.set_device(rank)
        ctx = sb.Context(rank)
        obj = [sb.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        ctx.tp_init(rank, world, obj[0])
        cfg, w = _weights(fmt, name)
        m = sb.Model(ctx, cfg, w, len(PROMPT) + STEPS + 8)
        tok, lg = m.forward_prefill(PROMPT)
        logits, toks = [lg], [tok]
        for _ in range(STEPS):
            nxt, lgs = m.forward_one([toks[-1]])
            toks.append(int(nxt[0]))
            logits.append(lgs[0])
        gen = None
        m.reset()
        m.forward_prefill(PROMPT, want_logits=False)
        gen = m.generate(STEPS)[0].tolist()
        if rank == 0:
            q.put((toks, np.stack(logits), gen))
        m.close()
        ctx.close()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("peer", ["0", "1"])  # NCCL collectives / the peer-memory kernel
@pytest.mark.parametrize("fmt,name", [("Q4_0", "tiny"), ("Q4_K", "tiny-k-tp")])
def test_tp2_model_matches_oracle(fmt, name, peer):
    import torch.multiprocessing as mp
    from oracle import oracle as O
    from oracle.lm import OracleLM
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, fmt, name, q, peer)) for r in range(2)]
    for p in procs:
        p.start()
    got = q.get(timeout=300)
    assert got[0] != "error", got
    toks, logits, gen = got
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    cfg, w = _weights(fmt, name)
    ref = OracleLM(cfg, w, len(PROMPT) + STEPS + 8)
    lref = ref.forward_prefill(PROMPT)
    assert gen == toks[1:]  # on-device generation == per-step API
    for i in range(STEPS + 1):
        err = np.linalg.norm(logits[i] - lref) / np.linalg.norm(lref)
        assert err < 5e-3, (i, err)
        if O.argmax(lref) != toks[i]:
            srt = np.sort(lref)
            # only where the oracle's top-2 margin is below the observed error
            assert srt[-1] - srt[-2] <= np.abs(logits[i] - lref).max(), i
            break
        if i < STEPS:
            lref = ref.forward_one(toks[i])


def _ar_rank(rank, world, port, q):
    import sys
    sys.path.insert(0, ROOT)
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port),
                      SYN_TP_PEER_ALLREDUCE="1")  # the peer-memory kernel (opt-in)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import synapse_b200 as sb
        torch.cuda.set_device(rank)
        ctx = sb.Context(rank)
        obj = [sb.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        ctx.tp_init(rank, world, obj[0])
        res = []
        for n in (4096, 1000 * 4, 3 << 18, 4096):  # peer path, peer, NCCL (large), peer again
            rng = np.random.default_rng(100 * n + rank)
            x = torch.from_numpy(rng.standard_normal(n).astype(np.float32)).cuda()
            for _ in range(3):  # repeated calls walk the double-buffered slots
                y = x.clone()
                ctx.tp_allreduce_sum(y)
            torch.cuda.synchronize()
            res.append(y.cpu().numpy())
        q.put((rank, res))
        ctx.close()
    except Exception as e:
        q.put(("error", rank, repr(e)))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp2_allreduce_sums_in_rank_order():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ar_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = [q.get(timeout=300) for _ in range(2)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert all(g[0] != "error" for g in got), got
    by = {g[0]: g[1] for g in got}
    for i, n in enumerate((4096, 4000, 3 << 18, 4096)):
        xs = [np.random.default_rng(100 * n + r).standard_normal(n).astype(np.float32)
              for r in range(2)]
        want = (np.float32(0) + xs[0]) + xs[1]
        assert np.array_equal(by[0][i], by[1][i]), n  # the same bits on every rank
        assert np.allclose(by[0][i], want, rtol=1e-6, atol=1e-6), n
