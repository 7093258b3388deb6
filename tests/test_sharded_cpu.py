"""Multi-process (gloo, world_size 2, CPU) tests of the row-sharded host
logic: shard planning, the amax exchange, global RNG coordinates, and a rank
that never joins.  The CUDA kernels are replaced by the oracle here (test
only); the same ShardedRhtQuantizer drives the kernels on GPUs."""
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _h16():
    sys.path.insert(0, str(ROOT))
    from oracle import oracle
    i = np.arange(16)
    par = np.array([[bin(a & b).count("1") & 1 for b in i] for a in i])
    return oracle.f32_to_bf16(np.where(par == 0, 0.25, -0.25).astype(np.float32))


def _worker(rank, world, port, mode, q):
    sys.path.insert(0, str(ROOT))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world))
    try:
        from datetime import timedelta
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=timedelta(seconds=3 if mode == "dropout" else 60))
        from fp4_sm120a_b200.sharded import ShardedRhtQuantizer, combine_amax
        from oracle import oracle
        m, n_total, kt = 128, 640, 128
        rng = np.random.default_rng(0)
        x = rng.standard_normal(m * n_total).astype(np.float32)
        if mode == "nan":
            x[m * 600 + 5] = np.nan      # lives in rank 1's shard
        A = oracle.f32_to_bf16(x)
        rs = (4242, 7)
        qz = ShardedRhtQuantizer(m, n_total, k_tile_size=kt, stochastic_rounding=True,
                                 rng_state=rs)
        lo, n = qz.n_offset, qz.n
        shard = torch.from_numpy(A[lo * m:(lo + n) * m].view(np.int16).copy())
        if mode == "dropout":
            if rank == 1:
                q.put((rank, "left"))
                return                   # never joins the exchange
            amax = torch.tensor([1.0])
            try:
                combine_amax(amax)
                q.put((rank, "no error"))
            except Exception as e:       # the collective must fail, not hang
                q.put((rank, "error:" + type(e).__name__))
            return

        def local_amax(a, out):
            out.fill_(oracle.amax_bf16(a.numpy().view(np.uint16)))

        def cast(qz_, a, B, C, S, amax):
            c, s = oracle.rht_gemm_ntt_w_sfc(qz_.m, qz_.n, a.numpy().view(np.uint16), B,
                                             float(amax.item()), rs, kt, True, False,
                                             qz_.n_offset, qz_.n_total)
            C.copy_(torch.from_numpy(c))
            S.copy_(torch.from_numpy(s))

        C, S = qz.outputs("cpu")
        amax = qz(shard, _h16(), C, S, local_amax_fn=local_amax, cast_fn=cast)
        Cs = [None] * world
        Ss = [None] * world
        dist.all_gather_object(Cs, C)      # shards differ in size (640 = 384 + 256)
        dist.all_gather_object(Ss, S)
        if rank == 0:
            full_amax = oracle.amax_bf16(A)
            if mode == "nan":
                q.put((rank, bool(np.isnan(amax.item())) and np.isnan(full_amax)))
                return
            Cf, Sf = oracle.rht_gemm_ntt_w_sfc(m, n_total, A, _h16(), full_amax, rs, kt, True,
                                               False)
            ok = (amax.item() == np.float32(full_amax)
                  and (torch.cat(Cs, 1).numpy() == Cf).all()
                  and (torch.cat(Ss, 1).numpy() == Sf).all())
            q.put((rank, bool(ok)))
        else:
            q.put((rank, bool(np.isnan(amax.item())) if mode == "nan" else True))
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, f"exception {type(e).__name__}: {e}"))
    finally:
        if dist.is_initialized() and mode != "dropout":
            dist.destroy_process_group()


def _run(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(2))
    for p in ps:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return res


def test_plan_shards_alignment():
    from fp4_sm120a_b200.sharded import plan_shards
    p = plan_shards(14336, 65536, 8)
    assert p.offsets == tuple(8192 * r for r in range(8)) and set(p.sizes) == {8192}
    p = plan_shards(256, 5120, 3)
    assert p.offsets == (0, 2048, 4096) and p.sizes == (2048, 2048, 1024)
    p = plan_shards(256, 320, 4, 128)
    assert sum(p.sizes) == 320 and all(o % 128 == 0 for o in p.offsets)
    with pytest.raises(ValueError):
        plan_shards(100, 320, 2)


def test_two_rank_sharded_equals_single():
    assert _run("ok") == {0: True, 1: True}


def test_two_rank_nan_amax_propagates():
    assert _run("nan") == {0: True, 1: True}


def test_rank_that_never_joins_times_out():
    res = _run("dropout")
    assert res[1] == "left"
    assert str(res[0]).startswith("error:")
