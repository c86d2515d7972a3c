"""GPU, 2 ranks (skipped with fewer than 2 GPUs): the output gathers into a mapped buffer.

Rank 0's output buffer is mapped into rank 1 (shard.PeerOutput: CUDA IPC, NVLink peer access).
"peer": each rank runs sage_run on its half of the heads with its output pointing into that
buffer, so rank 1's attention epilogue stores straight into rank 0's memory. "copy"
(shard.CopyGather): each rank computes its heads in waves on two alternating streams, rank 0
into its slice of the buffer and rank 1 into local memory, whose finished waves the copy engine
moves into the mapping. After a barrier, rank 0 holds the whole output, which must equal a
single-GPU run over all heads bit for bit. A second step into the same buffer checks that
nothing from the first leaks into it.
"""
import datetime
import os

import pytest
import torch

pytestmark = pytest.mark.gpu


def _rank_main(rank, world, port, case, results, mode="peer"):
    import torch.distributed as dist

    import tribench_b200 as tb
    from tribench_b200 import shard

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        B, H, S, D = case["batch_size"], case["num_heads"], case["seq_len"], case["head_dim"]
        sd = shard.make_shard(case, rank, world)
        peer = shard.PeerOutput((1, sd.total, S, D), torch.float16, 0, dev)
        ok = True
        for seed in (case["seed"], case["seed"] + 1):
            inp = tb.make_inputs(case, dev, seed=seed, dtype="fp16", heads=(sd.lo, sd.hi))
            n = sd.heads
            if mode == "peer":
                plan = tb.SagePlan(1, n, n, S, S, D, torch.float16, dev, causal=case["causal"])
                plan.run(inp["q"], inp["k"], inp["v"], peer.tensor[:, sd.lo:sd.hi])
            else:
                waves = shard.wave_ranges(sd.lo, sd.hi, 3)  # uneven waves: sizes 1 and 2 heads
                out = peer.tensor[:, sd.lo:sd.hi] if rank == 0 else torch.empty_like(inp["q"])
                plans = [{}, {}]

                def compute(a, b, slot):
                    m = b - a
                    pl = plans[slot].setdefault(m, tb.SagePlan(1, m, m, S, S, D, torch.float16, dev,
                                                                causal=case["causal"]))
                    i, j = a - sd.lo, b - sd.lo
                    pl.run(inp["q"][:, i:j], inp["k"][:, i:j], inp["v"][:, i:j], out[:, i:j])

                shard.CopyGather(peer, sd.lo, out).step(waves, compute)
            torch.cuda.synchronize(dev)
            dist.barrier()
            if rank == 0:
                full = tb.make_inputs(case, dev, seed=seed, dtype="fp16", heads=(0, sd.total))
                ref = tb.SagePlan(1, sd.total, sd.total, S, S, D, torch.float16, dev, causal=case["causal"]).run(
                    full["q"], full["k"], full["v"])
                ok = ok and torch.equal(peer.tensor, ref)
            dist.barrier()
        assert tb.device_status(dev) == 0
        peer.close()
        results.put((rank, ok))
    except Exception as e:  # reported to the parent
        results.put((rank, f"{type(e).__name__}: {e}"))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("mode", ["peer", "copy"])
def test_mapped_output_gather_matches_one_gpu_bit_for_bit(mode):
    import torch.multiprocessing as mp

    case = dict(batch_size=2, num_heads=4, seq_len=1000, head_dim=128, causal=True, dist="offset",
                k_offset_std=2.0, seed=5)
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = 29600 + os.getpid() % 200 + (7 if mode == "copy" else 0)
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, case, results, mode)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(results.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert got == {0: True, 1: True}, got
