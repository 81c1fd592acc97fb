"""GPU, two or more devices: the round-robin sharded separation over NCCL
(msst_b200.dist.ShardedSeparator) against one GPU's msst_model_separate, with
device-resident buffers and with host buffers (per-rank input windows, stitched
ranges copied down as they become final).  Runs as child processes, one per
GPU, with NVLink SHARP (NVLS) off; skipped on a one-GPU machine."""
from __future__ import annotations

import os
import socket
import sys

import numpy as np
import pytest

from conftest import PKG, ROOT, golden, snr_db

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, path, meta, out_path):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    sys.path.insert(0, PKG)
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    from msst_b200 import Model, synth
    from msst_b200.dist import ShardedSeparator

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, init_method=f"tcp://127.0.0.1:{port}",
                            timeout=timedelta(seconds=60), device_id=torch.device("cuda", rank))
    m = Model(path, rank, "fp16")
    track = synth.make_audio(meta["track_len"], 2, meta["track_seed"])
    dev = torch.from_numpy(track).cuda()
    sep = ShardedSeparator(m, dist, rank, world)
    y = sep.separate(dev, meta["overlap"], chunk_batch=2)
    y = y.cpu().numpy().copy() if rank == 0 else None
    pin_in = torch.from_numpy(track).pin_memory()
    pin_out = torch.full((1, 2, track.shape[1]), float("nan")).pin_memory() if rank == 0 else None
    scratch = torch.zeros_like(dev)
    sep.separate(scratch, meta["overlap"], chunk_batch=2, track_host=pin_in, out_host=pin_out)
    torch.cuda.synchronize()
    dist.barrier()
    if rank == 0:
        ref = m.separate(dev, meta["overlap"], chunk_batch=2).cpu().numpy()
        np.save(out_path, np.array([snr_db(y, ref), snr_db(pin_out.numpy()[0], ref),
                                    float(np.isfinite(pin_out.numpy()).all())]))
    m.close()
    dist.destroy_process_group()


def test_sharded_separation_nccl_matches_one_gpu(cuda, tmp_path):
    torch = cuda
    world = min(torch.cuda.device_count(), 4)
    if world < 2:
        pytest.skip("needs two GPUs")
    from msst_b200 import synth

    _, meta = golden("mbr_chunked_fp32.npz")
    cfg = synth.mbr_config(**meta["cfg"])
    path = str(tmp_path / "m.csm")
    synth.write_csm(path, cfg, synth.make_weights(cfg, meta["weights_seed"]))
    out = str(tmp_path / "res.npy")
    import torch.multiprocessing as tmp_mp

    ctx = tmp_mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, path, meta, out)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        if p.is_alive():
            p.kill()
            pytest.fail("a rank did not finish")
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    dev_snr, host_snr, finite = np.load(out)
    # batches differ from the one-GPU run (cuFFT picks batch-size-dependent plans)
    assert dev_snr >= 70.0 and host_snr >= 70.0 and finite == 1.0
