"""CPU, world size 2 over gloo: the (batch x head) partition and the wave-overlapped output
gather of tribench_b200.shard, including a rank that fails before sending its shard."""
import datetime
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from tribench_b200 import shard as sh

CASE = dict(batch_size=2, num_heads=5, seq_len=24, head_dim=64, dist="offset", k_offset_std=2.0)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _fake_attention(q, k, v):
    # stands in for the GPU kernel: any per-head function exercises the data movement
    return (q.float() * 0.5 + k.float() - v.float() * 0.25).to(q.dtype)


def _worker(rank, world, port, mode, results):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    try:
        sd = sh.make_shard(CASE, rank, world)
        inp = sh.shard_inputs(CASE, sd, "cpu", seed=3, dtype="fp16")
        B, H, S, D = CASE["batch_size"], CASE["num_heads"], CASE["seq_len"], CASE["head_dim"]
        full = torch.empty(B, H, S, D, dtype=torch.float16) if rank == 0 else None
        if mode == "alias" and rank == 0:
            # the destination computes straight into its slice of the full output (no copy)
            out = full.reshape(1, B * H, S, D)[:, sd.lo:sd.hi]
        else:
            out = torch.empty_like(inp["q"])

        def compute(a, b):
            i, j = a - sd.lo, b - sd.lo
            out[:, i:j] = _fake_attention(inp["q"][:, i:j], inp["k"][:, i:j], inp["v"][:, i:j])

        if mode == "fail" and rank == 1:
            raise RuntimeError("rank 1 fails before sending its shard")
        got = sh.gather_to(0, out, sd, full, waves=3, compute=compute, timeout_s=5.0)
        if rank == 0:
            ref_in = sh.make_inputs(CASE, "cpu", 3, "fp16")
            ref = _fake_attention(ref_in["q"], ref_in["k"], ref_in["v"])
            results.put(("ok", rank, bool(torch.equal(got, ref))))
        else:
            results.put(("ok", rank, True))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as exc:  # reported to the parent; the process then exits without teardown
        results.put(("error", rank, str(exc)[:200]))
        results.close()
        results.join_thread()  # flush the message before leaving
        os._exit(0)


def _run(mode):
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, results)) for r in range(2)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(2):
        kind, rank, val = results.get(timeout=120)
        out[rank] = (kind, val)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return out


def test_head_ranges_cover_grid_once():
    for total in (1, 7, 64, 1024):
        for world in (1, 2, 3, 8):
            seen = []
            sizes = []
            for r in range(world):
                lo, hi = sh.head_range(r, world, total)
                seen.extend(range(lo, hi))
                sizes.append(hi - lo)
            assert seen == list(range(total))
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        sh.head_range(2, 2, 10)


def test_wave_ranges():
    assert sh.wave_ranges(3, 10, 3) == [(3, 5), (5, 7), (7, 10)]
    assert sh.wave_ranges(0, 2, 5) == [(0, 1), (1, 2)]


def test_gather_world2_matches_single_process():
    out = _run("ok")
    assert out[0] == ("ok", True), out
    assert out[1][0] == "ok", out


def test_gather_into_aliased_destination_slice():
    out = _run("alias")
    assert out[0] == ("ok", True), out
    assert out[1][0] == "ok", out


def test_gather_rank_failure_is_reported_not_hung():
    out = _run("fail")
    assert out[1][0] == "error" and "fails before sending" in out[1][1]
    assert out[0][0] == "error", out  # rank 0's receive ends with an error at the group timeout
