"""CPU tests (no GPU) of the tensor-parallel split with world_size 2 over
gloo: every rank shards the weights with the library's host-side splitter
(syn_cuda_tp_shard_linear), computes its partial products with the oracle,
and the partials are combined the way the GPU ranks combine them (sum
all-reduce after row-parallel layers, all-gather after column-parallel /
vocabulary-parallel ones). The combined results must equal the unsharded
oracle: bit-exact for column splits, within f32 summation-order rounding for
row splits."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


CASES = [("Q4_0", 64, 256), ("Q8_0", 96, 128), ("Q4_K", 64, 1024), ("Q6_K", 32, 512),
         ("INT8_KN", 64, 96)]


def _worker(rank, world, port, q):
    import sys
    sys.path.insert(0, ROOT)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        out = [_case(rank, world, *c) for c in CASES]
        if rank == 0:
            q.put(out)
    finally:
        dist.destroy_process_group()


def _case(rank, world, fmt, n, k):
    if True:
        import synapse_b200 as sb
        from synapse_b200 import synth
        from oracle import oracle as O
        rng = np.random.default_rng(42)
        data, scales = synth.gen_weight(sb.QFormat[fmt], n, k, rng)
        x = synth.gen_activations(3, k, rng)

        def matmul(d, nn, kk, xx, sc):
            if fmt == "INT8_KN":
                st, xq, sx = O.quantize_per_channel_int8(xx, xx.shape[0], kk)
                return O.naive_int8_gemm(xx.shape[0], nn, kk, xq, d.view(np.int8), sx,
                                         sc).reshape(-1, nn)
            st, y = O.block_matmul(fmt, xx.shape[0], nn, kk, np.ascontiguousarray(xx), d)
            assert st == 0
            return y.reshape(-1, nn)

        full = matmul(data, n, k, x, scales)
        res = {}
        # column-parallel (axis 0): all-gather of the output slices
        d0, n0, k0, s0 = sb.tp_shard_linear(fmt, data, n, k, rank, world, 0, scales)
        assert (n0, k0) == (n // world, k)
        part = torch.from_numpy(matmul(d0, n0, k0, x, s0).copy())
        gathered = [torch.empty_like(part) for _ in range(world)]
        dist.all_gather(gathered, part)
        res["col"] = torch.cat(gathered, dim=1).numpy()
        if fmt != "INT8_KN":
            # row-parallel (axis 1): x split along K, sum all-reduce
            d1, n1, k1, _ = sb.tp_shard_linear(fmt, data, n, k, rank, world, 1, scales)
            assert (n1, k1) == (n, k // world)
            xs = np.ascontiguousarray(x[:, rank * k1:(rank + 1) * k1])
            t = torch.from_numpy(matmul(d1, n1, k1, xs, None).copy())
            dist.all_reduce(t)
            res["row"] = t.numpy()
        # vocabulary-parallel argmax: gather logits in rank order
        logits = rng.standard_normal(4 * world * 8).astype(np.float32)
        logits[[5, 37]] = 9.0  # a tie across ranks: the later index wins
        sl = torch.from_numpy(logits.reshape(world, -1)[rank].copy())
        g2 = [torch.empty_like(sl) for _ in range(world)]
        dist.all_gather(g2, sl)
        res["argmax"] = (O.argmax(torch.cat(g2).numpy()), O.argmax(logits))
        return fmt, full, res


def test_tp2_shards_recombine_to_the_unsharded_result():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = q.get(timeout=300)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert [o[0] for o in out] == [c[0] for c in CASES]
    for fmt, full, res in out:
        assert np.array_equal(res["col"], full), fmt
        if "row" in res:
            np.testing.assert_allclose(res["row"], full, rtol=1e-4,
                                       atol=1e-4 * np.abs(full).max(), err_msg=fmt)
        assert res["argmax"][0] == res["argmax"][1], fmt
