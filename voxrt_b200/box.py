"""Box-level scheduling of many utterances over the GPUs of one node: one encoder replica per GPU, no collective.

Every utterance's encoder forward is independent, so a batch of utterances is partitioned, not exchanged:

  * ``lpt_shards``     longest-processing-time-first assignment of utterances to GPUs on the cost
                       T + T^2 / 1500 encoder frames (the GEMMs grow with T, the attention with T^2);
  * ``length_buckets`` each GPU's utterances, longest first, cut into runs of at most ``budget`` encoder frames;
                       each run is one token-stacked forward (an utterance longer than the budget runs alone);
  * ``RankPipeline``   one GPU's share: the bucketed forwards, the frames of every bucket gathered into the
                       caller's per-utterance host slots, and (optionally) the TDT decode: all of the rank's
                       utterances in one lockstep batch on the GPU after the forwards, or bucket b on host threads
                       while the GPU encodes bucket b + 1 (the two-stage encoder/decoder pipeline of
                       Transcriber::transcribe_long, crates/voxrt/src/transcriber.rs:356-386, with buckets in the
                       role of its VAD segments);
  * ``BoxEncoder``     the same in one process: a RankPipeline per device, each on its own host thread.

Processes launched one per GPU (torchrun) call ``plan(..., world)[rank]`` and run a ``RankPipeline`` each; the
host gather is per rank. All arithmetic runs in libvxg.so's kernels through the encoder's C ABI.
"""
from __future__ import annotations

import threading
import time

import numpy as np

ATTN_COST_FRAMES = 1500.0  # T at which a frame's attention work equals its GEMM work in the cost model
DEFAULT_BUDGET = 131072    # encoder frames per token-stacked forward


def cost(te) -> np.ndarray:
    te = np.asarray(te, np.float64)
    return te + te ** 2 / ATTN_COST_FRAMES


def lpt_shards(te, world: int) -> list[list[int]]:
    """Utterance ids per rank: longest first onto the least-loaded rank; each rank's list sorted longest first."""
    te = np.asarray(te, np.int64)
    if world < 1:
        raise ValueError("world must be >= 1")
    c = cost(te)
    load = np.zeros(world)
    shards: list[list[int]] = [[] for _ in range(world)]
    for u in np.argsort(-c, kind="stable"):
        r = int(np.argmin(load))
        shards[r].append(int(u))
        load[r] += c[u]
    return [sorted(s, key=lambda u: (-te[u], u)) for s in shards]


def length_buckets(order, te, budget: int = DEFAULT_BUDGET) -> list[list[int]]:
    """Consecutive runs of `order` (length-sorted utterance ids) holding at most `budget` encoder frames each."""
    te = np.asarray(te, np.int64)
    out, cur, tot = [], [], 0
    for u in order:
        if cur and tot + te[u] > budget:
            out.append(cur)
            cur, tot = [], 0
        cur.append(int(u))
        tot += int(te[u])
    if cur:
        out.append(cur)
    return out


def plan(t_in, world: int, budget: int = DEFAULT_BUDGET, out_frames=None) -> list[list[list[int]]]:
    """Buckets of utterance ids for each of `world` ranks, from the utterances' log-mel frame counts."""
    if out_frames is None:
        from .encoder import CudaEncoder

        out_frames = CudaEncoder.out_frames
    te = np.array([out_frames(int(t)) for t in t_in], np.int64)
    return [length_buckets(s, te, budget) for s in lpt_shards(te, world)]


class RankPipeline:
    """One GPU's share of a box workload (see the module docstring).

    encoder: a CudaEncoder on this rank's device; decoder: an optional TdtDecoder created for the same device (its
    encoder projection and batched greedy decode run there; the host greedy loop uses `decode_threads` threads).
    second_encoder: an optional second CudaEncoder of the same model on the same device; with it, encode() keeps
    two host-buffer calls in flight (alternate buckets on two host threads), so one bucket's host <-> device copies
    overlap the other bucket's kernels."""

    def __init__(self, encoder, decoder=None, decode_threads: int = 0, second_encoder=None):
        self.enc = encoder
        self.dec = decoder
        self.decode_threads = decode_threads
        self.enc2 = second_encoder

    def encode(self, feats, buckets, outs=None, stream=None):
        """Encoder frames of every utterance in `buckets` (lists of ids into `feats`), through the host-buffer C ABI
        entry (one token-stacked forward per bucket, host feats in, host frames out into outs[u]). Returns outs
        (a dict id -> [t_e, d] array; arrays the caller passes are reused)."""
        outs = {} if outs is None else outs

        def run(enc, bks):
            for b in bks:
                fb = [feats[u] for u in b]
                slot = [outs.get(u) for u in b]
                if any(s is None for s in slot):
                    slot = [np.empty((enc.out_frames(f.shape[0]), enc.d_model), np.float32) for f in fb]
                enc.forward_batch(fb, slot)
                for u, s in zip(b, slot):
                    outs[u] = s

        if self.enc2 is None or len(buckets) < 2:
            run(self.enc, buckets)
            return outs
        from concurrent.futures import ThreadPoolExecutor

        with ThreadPoolExecutor(2) as ex:  # the library releases the GIL inside each call
            jobs = [ex.submit(run, e, buckets[i::2]) for i, e in enumerate((self.enc, self.enc2))]
            for j in jobs:
                j.result()
        return outs

    def encode_device(self, feats_dev, t_in_b, outs_dev, stream=None):
        """Device-resident forwards: feats_dev[i] / outs_dev[i] are the i-th bucket's stacked torch CUDA tensors.
        Returns the list of (start, end) CUDA events of the forwards, recorded on the current stream."""
        import torch

        evs = []
        for fd, tb, od in zip(feats_dev, t_in_b, outs_dev):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            self.enc.forward_device(fd, tb, od)
            e1.record()
            evs.append((e0, e1))
        return evs

    def transcribe(self, feats, buckets, decode: str = "gpu", timings: dict | None = None):
        """Encoder + TDT greedy decode of every utterance in `buckets`; returns {id: emissions [n, 3] int32}.

        decode="gpu": every bucket's forward and encoder projection run back to back into one device buffer of
        projected frames; then all utterances are decoded together in lockstep rounds on the GPU
        (TdtDecoder.greedy_device). The decode's rounds are many small latency-bound launches, so they run with the
        GPU to themselves rather than queued behind the encoder's persistent GEMMs, and the one batch serves the
        whole rank's utterances per pass over the decoder weights. decode="host": the two-stage pipeline of
        Transcriber::transcribe_long (transcriber.rs:370-386) -- bucket b's projected frames decoded on host threads
        (greedy_batch) while the GPU encodes bucket b + 1. Both give identical emissions. With decode="gpu",
        `timings` (a dict) receives the wall seconds of the encode and decode phases."""
        import torch

        assert self.dec is not None, "no decoder"
        assert decode in ("gpu", "host")
        dev = self.enc.device
        te_all = {u: self.enc.out_frames(feats[u].shape[0]) for b in buckets for u in b}
        if decode == "gpu":
            t0 = time.perf_counter()
            order = [u for b in buckets for u in b]
            frames = [te_all[u] for u in order]
            proj = torch.empty((int(sum(frames)), self.dec.hidden), dtype=torch.float32, device=f"cuda:{dev}")
            # bucket b's feats are gathered into one of two page-locked buffers and copied on a copy stream into one
            # of two device buffers, so the host prepares bucket b + 1 and the copy engine moves it while the GPU
            # encodes bucket b
            n_mels = feats[order[0]].shape[1] if order else 0
            most = max((sum(feats[u].shape[0] for u in b) for b in buckets), default=0)
            cuda = f"cuda:{dev}"
            pin = [torch.empty((most, n_mels), dtype=torch.float32, pin_memory=True) for _ in range(2)]
            fdev = [torch.empty((most, n_mels), dtype=torch.float32, device=cuda) for _ in range(2)]
            copy_stream = torch.cuda.Stream(device=cuda)
            compute = torch.cuda.current_stream(cuda)
            copied: list = [None, None]  # copy into buffer k done (copy stream)
            read: list = [None, None]    # forward that read device buffer k done (compute stream)
            row = 0
            for i, b in enumerate(buckets):
                fb = [feats[u] for u in b]
                n = int(sum(te_all[u] for u in b))
                rows_in = int(sum(f.shape[0] for f in fb))
                k = i & 1
                if copied[k] is not None:
                    copied[k].synchronize()  # the copy that last read this page-locked buffer is done
                np.concatenate(fb, out=pin[k][:rows_in].numpy())
                with torch.cuda.stream(copy_stream):
                    if read[k] is not None:
                        copy_stream.wait_event(read[k])
                    fdev[k][:rows_in].copy_(pin[k][:rows_in], non_blocking=True)
                    copied[k] = torch.cuda.Event()
                    copied[k].record(copy_stream)
                compute.wait_event(copied[k])
                out = torch.empty((n, self.enc.d_model), dtype=torch.float32, device=cuda)
                self.enc.forward_device(fdev[k][:rows_in], np.array([f.shape[0] for f in fb], np.int32), out)
                self.dec.project_device(out, out=proj[row:row + n])
                read[k] = torch.cuda.Event()
                read[k].record(compute)
                row += n
            if timings is not None:
                torch.cuda.synchronize(dev)
                t1 = time.perf_counter()
            res = dict(zip(order, self.dec.greedy_device(proj, frames, timings=timings)))
            if timings is not None:
                timings["encode_s"] = t1 - t0
                timings["decode_s"] = time.perf_counter() - t1
            return res
        results = {}
        errors: list[BaseException] = []
        pending = None
        for b in buckets:
            fb = [feats[u] for u in b]
            te = [te_all[u] for u in b]
            fd = torch.from_numpy(np.concatenate(fb)).to(f"cuda:{dev}", non_blocking=False)
            out = torch.empty((int(sum(te)), self.enc.d_model), dtype=torch.float32, device=fd.device)
            self.enc.forward_device(fd, np.array([f.shape[0] for f in fb], np.int32), out)
            proj = self.dec.project_device(out).cpu()  # waits for this bucket's encoder
            if pending is not None:
                pending.join()

            def work(bb=b, pp=proj, tt=te):
                try:
                    offs = np.concatenate([[0], np.cumsum(tt)])
                    parts = [pp[offs[i]:offs[i + 1]].numpy() for i in range(len(bb))]
                    for u, r in zip(bb, self.dec.greedy_batch(parts, threads=self.decode_threads)):
                        results[u] = r
                except BaseException as ex:  # re-raised on the calling thread
                    errors.append(ex)

            pending = threading.Thread(target=work)
            pending.start()
        if pending is not None:
            pending.join()
        if errors:
            raise errors[0]
        return results


class BoxEncoder:
    """All GPUs of the node from one process: a CudaEncoder per device, utterances LPT-sharded over them, each
    device's share run by a RankPipeline on its own host thread; outputs gathered on the host."""

    def __init__(self, model: dict, devices, weights: str = "2bit", budget: int = DEFAULT_BUDGET):
        from .encoder import CudaEncoder

        self.devices = list(devices)
        self.budget = budget
        self.pipes = [RankPipeline(CudaEncoder.load(model, device=d, weights=weights)) for d in self.devices]

    def close(self):
        for p in self.pipes:
            p.enc.close()

    def encode(self, feats) -> tuple[list[np.ndarray], float]:
        """Encoder frames of every utterance (host arrays in, host arrays out, in input order) and the wall time."""
        import torch

        plans = plan([f.shape[0] for f in feats], len(self.pipes), self.budget)
        results: list[dict] = [dict() for _ in self.pipes]
        errors: list[BaseException] = []

        def work(i):
            try:
                torch.cuda.set_device(self.devices[i])
                self.pipes[i].encode(feats, plans[i], results[i])
            except BaseException as ex:  # reported to the caller below
                errors.append(ex)

        t0 = time.perf_counter()
        th = [threading.Thread(target=work, args=(i,)) for i in range(len(self.pipes))]
        for t in th:
            t.start()
        for t in th:
            t.join()
        wall = time.perf_counter() - t0
        if errors:
            raise errors[0]
        merged = {}
        for r in results:
            merged.update(r)
        return [merged[u] for u in range(len(feats))], wall
