"""Chunk-sharded separation of one track over the GPUs of a node.

The reference separates a track chunk by chunk on one GPU
(src/inference_app.cpp:100-324).  Chunks carry no state between each other, so
here the chunk list of the whole plan is dealt out round-robin: rank r runs
chunks r, r + W, r + 2W, ... (W = world size), chunk_batch of them per forward
(msst_model_forward_chunks_strided).  After every forward batch each rank sends
its chunk outputs to rank 0 (one grouped NCCL send / receive per round), and rank
0 overlap-adds every output sample as soon as all the chunks that touch it have
arrived (msst_model_stitch_range), in chunk order, so the stitched track is the
single-GPU msst_model_separate result.  Because round j completes the chunk prefix
[0, (j+1) * chunk_batch * W), the stitched output grows as a prefix: with host
buffers it is copied down range by range while later rounds still compute, and
every rank copies up only the track samples its own chunks read.

Rank 0 stitches round j after enqueuing round j + 1's forward, so its stream waits
for round j's receives only once that forward is done; the transfers themselves
run on the communication stream while the ranks compute.

The compute functions are injectable so the sharding and gather logic can be
exercised with CPU tensors on a gloo process group.
"""
from __future__ import annotations


def shard(num_chunks: int, world: int, rank: int) -> tuple[int, int]:
    """(first chunk, count) of `rank` under round-robin dealing (stride = world)."""
    count = len(range(rank, num_chunks, world))
    return rank, count


def max_shard(num_chunks: int, world: int) -> int:
    return -(-num_chunks // world)


def round_chunks(num_chunks: int, world: int, rank: int, chunk_batch: int, rnd: int) -> list[int]:
    """Chunk indices `rank` runs in forward round `rnd`."""
    mine = list(range(rank, num_chunks, world))
    return mine[rnd * chunk_batch:(rnd + 1) * chunk_batch]


class ShardedSeparator:
    """Separate one track with its chunks dealt out over the ranks of a process group.

    model:          msst_b200.Model on this rank's GPU (default compute), or None
    dist:           torch.distributed (initialised), or None for a single process
    forward:        fn(track, overlap, first, stride, count, chunk_batch, fix_tail_padding, out) -> out
    stitch_range:   fn(chunks, slot_ranks, slot_cap, C, L, overlap, begin, end, out) -> out
    plan:           fn(L, overlap) -> dict(num_chunks=..., chunk_size=...)
    span:           fn(L, overlap, k, fix_tail_padding) -> ([(in_begin, in_end), ...], (out_begin, out_end))
    stems:          number of stems (from the model by default)
    """

    def __init__(self, model=None, dist=None, rank: int = 0, world: int = 1, forward=None, stitch_range=None,
                 plan=None, span=None, stems: int | None = None):
        self.model = model
        self.dist = dist
        self.rank = rank
        self.world = world
        self._forward = forward or (lambda track, overlap, first, stride, count, cb, fix, out:
                                    model.forward_chunks_strided(track, overlap, first, stride, count, cb, fix,
                                                                 out=out))
        self._stitch_range = stitch_range or (lambda chunks, sr, sc, C, L, overlap, b, e, out: model.stitch_range(
            chunks, sr, sc, C, L, overlap, b, e, out))
        self._plan = plan or (lambda L, overlap: model.chunk_plan(L, overlap))
        self._span = span or (lambda L, overlap, k, fix: model.chunk_span(L, overlap, k, fix))
        self.stems = stems if stems is not None else model.info["num_stems"]
        self._bufs = {}
        self.last_h2d_bytes = 0
        self.last_d2h_bytes = 0
        # profile=True: CUDA events split the next separate() into this rank's own
        # forwards (start -> last forward queued) and the tail after them (waiting
        # for the last round's transfers, the final stitch and copies): last_profile
        self.profile = False
        self.last_profile = None

    def _buffer(self, name, shape, like):
        import torch

        b = self._bufs.get(name)
        if b is None or tuple(b.shape) != tuple(shape) or b.device != like.device:
            b = torch.empty(shape, dtype=torch.float32, device=like.device)
            self._bufs[name] = b
        return b

    def _stream(self, name, device):
        import torch

        key = (name, str(device))
        st = self._bufs.get(key)
        if st is None:
            st = self._bufs[key] = torch.cuda.Stream(device=device)
        return st

    def separate(self, track, overlap: float = 0.0, chunk_batch: int = 0, fix_tail_padding: bool = False,
                 track_host=None, out_host=None):
        """track [C, L] device buffer on every rank -> stems [S, C, L] on rank 0, None on the others.

        track_host: optional host [C, L] array (pinned for asynchronous copies); only the
        samples this rank's chunks read are copied into `track`, piece by piece on a side
        stream, each forward waiting for its own piece.  out_host (rank 0): host [S, C, L]
        array that receives every stitched range as soon as it is final.
        """
        import torch

        C, L = track.shape
        W, r = self.world, self.rank
        plan = self._plan(L, overlap)
        n, chunk = plan["num_chunks"], plan["chunk_size"]
        cb = max(1, chunk_batch if chunk_batch > 0 else 2)
        cap = max_shard(n, W)
        rounds = -(-cap // cb)
        rows = self.stems * C
        is_cuda = track.device.type == "cuda"
        if r == 0:
            allbuf = self._buffer("all", (W * cap, rows, chunk), track)
            local = allbuf[:cap]
            out = self._buffer("out", (self.stems, C, L), track)
        else:
            local = self._buffer("local", (cap, rows, chunk), track)
            out = None
        self.last_h2d_bytes = self.last_d2h_bytes = 0

        # ---- host track: this rank's pieces, one per forward round, on an upload stream
        up_events = []
        if track_host is not None:
            up = self._stream("up", track.device) if is_cuda else None
            if is_cuda:
                up.wait_stream(torch.cuda.current_stream(track.device))
            host = torch.from_numpy(track_host) if not torch.is_tensor(track_host) else track_host
            for j in range(rounds):
                spans = [sp for k in round_chunks(n, W, r, cb, j) for sp in self._span(L, overlap, k,
                                                                                        fix_tail_padding)[0]]
                with torch.cuda.stream(up) if is_cuda else _nullctx():
                    for lo, hi in _merge(spans):
                        for c in range(C):
                            track[c, lo:hi].copy_(host[c, lo:hi], non_blocking=is_cuda)
                        self.last_h2d_bytes += 4 * C * (hi - lo)
                    if is_cuda:
                        ev = torch.cuda.Event()
                        ev.record(up)
                        up_events.append(ev)

        down = None
        if out_host is not None and r == 0 and is_cuda:
            down = self._stream("down", track.device)
        host_out = None
        if out_host is not None and r == 0:
            host_out = torch.from_numpy(out_host) if not torch.is_tensor(out_host) else out_host

        state = {"done": 0}

        def stitch_upto(k_done):
            """Rank 0: stitch every sample that chunks >= k_done do not touch."""
            upto = L if k_done >= n else self._span(L, overlap, k_done, fix_tail_padding)[1][0]
            b = state["done"]
            if upto <= b:
                return
            self._stitch_range(allbuf, W, cap, C, L, overlap, b, upto, out)
            if host_out is not None:
                flat_out, flat_host = out.view(rows, L), host_out.view(rows, L)
                if down is not None:
                    down.wait_stream(torch.cuda.current_stream(track.device))
                    with torch.cuda.stream(down):
                        for q in range(rows):
                            flat_host[q, b:upto].copy_(flat_out[q, b:upto], non_blocking=True)
                else:
                    flat_host[:, b:upto].copy_(flat_out[:, b:upto])
                self.last_d2h_bytes += 4 * rows * (upto - b)
            state["done"] = upto

        pending = []  # rank 0: (round, works) not yet stitched
        sends = []
        prof = None
        if self.profile and is_cuda:
            prof = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
            prof[0].record()
        for j in range(rounds):
            mine = round_chunks(n, W, r, cb, j)
            if up_events:
                torch.cuda.current_stream(track.device).wait_event(up_events[j])
            if mine:
                self._forward(track, overlap, mine[0], W, len(mine), cb, fix_tail_padding,
                              local[j * cb:j * cb + len(mine)])
            if prof is not None and j == rounds - 1:
                prof[1].record()
            works = []
            if W > 1:
                ops = []
                if r == 0:
                    for src in range(1, W):
                        cnt = len(round_chunks(n, W, src, cb, j))
                        if cnt:
                            ops.append(self.dist.P2POp(self.dist.irecv,
                                                       allbuf[src * cap + j * cb:src * cap + j * cb + cnt], src))
                elif mine:
                    ops.append(self.dist.P2POp(self.dist.isend, local[j * cb:j * cb + len(mine)], 0))
                if ops:
                    works = self.dist.batch_isend_irecv(ops)
            if r == 0:
                # stitch the previous round now that this round's forward is queued
                for pj, pw in pending:
                    for w in pw:
                        w.wait()
                    stitch_upto(min(n, (pj + 1) * cb * W))
                pending = [(j, works)]
            else:
                sends.extend(works)
        for w in sends:
            w.wait()
        if r == 0:
            for pj, pw in pending:
                for w in pw:
                    w.wait()
            stitch_upto(n)
            if down is not None:
                torch.cuda.current_stream(track.device).wait_stream(down)
        if prof is not None:
            prof[2].record()
            prof[2].synchronize()
            self.last_profile = {"forward_ms": prof[0].elapsed_time(prof[1]),
                                 "tail_ms": prof[1].elapsed_time(prof[2])}
        if r != 0:
            return None
        return out[0] if self.stems == 1 else out


class _nullctx:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


def _merge(spans):
    """Union of [lo, hi) ranges as sorted disjoint ranges."""
    out = []
    for lo, hi in sorted(spans):
        if out and lo <= out[-1][1]:
            out[-1][1] = max(out[-1][1], hi)
        else:
            out.append([lo, hi])
    return [(a, b) for a, b in out]
