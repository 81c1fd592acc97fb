"""CPU: chunk-sharded separation (msst_b200.dist.ShardedSeparator) over gloo ranks.

The compute is the fp32 oracle on CPU tensors; what is tested is the round-robin
dealing, the per-round sends to rank 0, the round-robin slot layout and the
progressive in-order stitch (range by range, copied into a host output as each
range becomes final): the sharded result must be bit-identical to
single-process separation.  A second test kills a rank before the first round's
transfer and checks that the survivor fails with an error within the
process-group timeout instead of hanging.
"""
from __future__ import annotations

import os
import socket
import sys

import numpy as np
import pytest

from conftest import PKG, ROOT

CHUNK = 22050


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _setup():
    for p in (PKG, os.path.join(ROOT, "oracle")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import oracle
    from msst_b200 import synth

    oracle.set_threads(2)
    cfg = synth.mbr_config(depth=1, dim=128, chunk_size=CHUNK)
    om = oracle.Model(cfg, synth.make_weights(cfg, 13))
    track = synth.make_audio(3 * CHUNK + 777, 2, 6)
    return oracle, om, track


def _worker(rank, world, port, out_path, fail_rank):
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    oracle, om, track = _setup()
    from msst_b200.dist import ShardedSeparator

    dist.init_process_group("gloo", rank=rank, world_size=world, init_method=f"tcp://127.0.0.1:{port}",
                            timeout=timedelta(seconds=10))
    step = oracle.resolve_step(CHUNK, 0.25, 2)
    inputs = oracle.chunk_inputs(track, CHUNK, step)
    border, total, starts = oracle.chunk_plan(track.shape[1], CHUNK, step)

    def plan(L, overlap):
        return dict(num_chunks=len(starts), chunk_size=CHUNK)

    def span(L, overlap, k, fix):
        s0, e0 = starts[k], min(starts[k] + CHUNK, total)
        return [(0, L)], (min(max(s0 - border, 0), L), min(max(e0 - border, 0), L))

    def fwd(trk, overlap, first, stride, count, cb, fix, out):
        for i in range(count):
            out[i] = torch.from_numpy(om.forward(inputs[first + i * stride][None])[0])
        return out

    def stitch_range(chunks, sr, sc, C, L, overlap, b, e, out):
        ys = [chunks[(k % sr) * sc + k // sr].numpy() for k in range(len(starts))]
        full = oracle.stitch(ys, L, CHUNK, step)
        out[0, :, b:e] = torch.from_numpy(full[:, b:e])
        return out

    sep = ShardedSeparator(None, dist, rank, world, fwd, stitch_range, plan, span, stems=1)
    sep._bufs["all"] = torch.zeros((world * -(-len(starts) // world), 2, CHUNK))
    try:
        if rank == fail_rank:
            raise SystemExit(3)  # this rank dies before the first round's transfer
        host_out = np.full((1, 2, track.shape[1]), np.nan, np.float32) if rank == 0 else None
        y = sep.separate(torch.zeros(track.shape), overlap=0.25, chunk_batch=1, track_host=track,
                         out_host=host_out)
        if rank == 0:
            ref = oracle.separate(lambda a: om.forward(a), track, CHUNK, step, batch=4)
            diff = max(float(np.abs(y.numpy() - ref).max()), float(np.abs(host_out[0] - ref).max()))
            np.save(out_path, np.array([diff, float(y.shape[1])]))
        dist.destroy_process_group()
    except RuntimeError as e:  # collective failed because a peer is gone
        if rank == 0:
            with open(out_path + ".err", "w") as f:
                f.write(str(e)[:500])


def _run(world, fail_rank, tmp_path):
    import torch.multiprocessing as tmp_mp

    out = str(tmp_path / f"res_{world}_{fail_rank}.npy")
    port = _free_port()
    ctx = tmp_mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, world, port, out, fail_rank)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
        if p.is_alive():
            p.kill()
            pytest.fail("a rank hung")
    return out


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_separation_matches_single_process(tmp_path, world):
    out = _run(world, -1, tmp_path)
    diff, length = np.load(out)
    assert length == 3 * CHUNK + 777
    assert diff == 0.0


def test_rank_failure_is_reported_not_hung(tmp_path):
    out = _run(2, 1, tmp_path)
    assert os.path.exists(out + ".err"), "surviving rank did not observe the failure"


def test_shard_ranges():
    from msst_b200.dist import max_shard, round_chunks, shard

    for n in (1, 5, 13, 92, 101):
        for w in (1, 2, 3, 8):
            spans = [shard(n, w, r) for r in range(w)]
            assert sum(c for _, c in spans) == n
            assert max(c for _, c in spans) - min(c for _, c in spans) <= 1
            assert max(c for _, c in spans) == max_shard(n, w)
            for cb in (1, 4):
                # round j of all ranks together covers the chunk prefix [j*cb*w, (j+1)*cb*w)
                rounds = -(-max_shard(n, w) // cb)
                for j in range(rounds):
                    got = sorted(k for r in range(w) for k in round_chunks(n, w, r, cb, j))
                    assert got == list(range(j * cb * w, min(n, (j + 1) * cb * w)))
