"""Row-sharded quantization on 2 GPUs over NCCL (skipped with fewer GPUs):
each rank quantizes its column shard after the int32-MAX amax exchange; the
gathered shards must equal a single-GPU run of the whole matrix bit for bit."""
import os
import socket
import sys
from pathlib import Path

import pytest
import torch
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent
pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q, exchange="nccl", mode="ok", fused=False):
    sys.path.insert(0, str(ROOT))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    try:
        import torch.distributed as dist
        from fp4_sm120a_b200 import ops
        from fp4_sm120a_b200.sharded import ShardedRhtQuantizer, init_distributed
        init_distributed("nccl", timeout_s=60)
        m, n_total = 1024, 8192
        g = torch.Generator(device="cuda").manual_seed(7)
        A = (torch.randn(m * n_total, device="cuda", generator=g) * 2).to(torch.bfloat16)
        B = ops.hadamard16(device="cuda")
        rs = torch.tensor([99, 3], dtype=torch.int64, device="cuda")
        qz = ShardedRhtQuantizer(m, n_total, k_tile_size=2048, rng_state=rs, exchange=exchange,
                                 fused=fused)
        shard = A[qz.n_offset * m:(qz.n_offset + qz.n) * m]
        C, S = qz.outputs()
        if mode == "dropout":
            # rank 1 stays out of one step (no kernel of its in flight); rank 0's
            # kernel must give up waiting for its amax and report it.
            if rank == 0:
                qz(shard, B, C, S)
                torch.cuda.synchronize()
                q.put((rank, ops.device_error()))
            else:
                q.put((rank, "skipped"))
            dist.barrier()
            dist.destroy_process_group()
            return
        if mode == "side_stream":
            # the step runs on a stream that is not torch's current one, which
            # is kept busy first: the all-reduce must still sit between the
            # amax kernel and the cast on that stream
            side = torch.cuda.Stream()
            with torch.cuda.stream(side):
                busy = torch.randn(1 << 27, device="cuda")
                for _ in range(20):
                    busy.mul_(1.0001)
            for _ in range(3):
                amax = qz(shard, B, C, S, stream=side)
            torch.cuda.current_stream().wait_stream(side)
        else:
            for _ in range(3):      # several steps: epochs advance, slots alternate
                amax = qz(shard, B, C, S)
        Cs = [torch.empty((m, sz // 2), dtype=torch.uint8, device="cuda") for sz in qz.plan.sizes]
        Ss = [torch.empty((m, sz // 16), dtype=torch.uint8, device="cuda") for sz in qz.plan.sizes]
        dist.all_gather(Cs, C)
        dist.all_gather(Ss, S)
        ok = True
        if rank == 0:
            Cf = torch.empty((m, n_total // 2), dtype=torch.uint8, device="cuda")
            Sf = torch.empty((m, n_total // 16), dtype=torch.uint8, device="cuda")
            am = torch.empty(1, device="cuda")
            ops.amax_bf16(A, m * n_total, am)
            ops.rht_gemm_ntt_w_sfc(m, n_total, A, B, Cf, Sf, am, rs, 0, None, 2048,
                                   stochastic_rounding=True)
            ok = (torch.equal(am, amax) and torch.equal(torch.cat(Cs, 1), Cf)
                  and torch.equal(torch.cat(Ss, 1), Sf))
        q.put((rank, bool(ok)))
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover
        q.put((rank, f"{type(e).__name__}: {e}"))


def _run(exchange, mode="ok", fused=False):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q, exchange, mode, fused)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(2))
    for p in ps:
        p.join(timeout=60)
    return res


@pytest.mark.parametrize("exchange,fused", [("nccl", False), ("peer", False), ("peer", True)])
def test_two_gpu_sharded_equals_single_gpu(exchange, fused):
    res = _run(exchange, fused=fused)
    assert res == {0: True, 1: True}, res


def test_peer_exchange_gives_up_when_a_rank_does_not_join():
    res = _run("peer", "dropout")
    assert res[1] == "skipped"
    assert res[0] == 5, res     # kErrTimeoutExchange, recorded instead of a hang


def test_two_gpu_nccl_exchange_on_a_non_current_stream():
    res = _run("nccl", "side_stream")
    assert res == {0: True, 1: True}, res
