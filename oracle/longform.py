"""LongForm (crates/voxrt/src/longform.rs) restated in Python, in its collect-only mode: the ranges of the segments
the streaming state machine closes, for a given VAD-probability function of an audio block.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py). `block_probs(samples, skip, want)` returns the probabilities of
frames [skip, skip + want) of the block (vad_block_at's last three lines, longform.rs:111-114); segment() is the
oracle's restatement of vad.rs:140-240.
"""
from __future__ import annotations

from . import SEGMENT_DEFAULTS, segment


class LongFormOracle:
    """LongForm::new / push / flush / drain / emit (longform.rs:29-193) with collect_only = true."""

    def __init__(self, block_probs, seg_cfg=None, block_samples=160000, ctx_samples=16 * 1280, spf=1280):
        self.block_probs = block_probs
        self.cfg = dict(SEGMENT_DEFAULTS, **(seg_cfg or {}))
        self.block_samples, self.ctx_samples, self.spf = block_samples, ctx_samples, spf
        self.pending = []        # audio from base_sample onward (a list of float32 values)
        self.base_sample = 0
        self.probs = []
        self.next_block = 0
        self.total = 0
        self.ranges = []
        self.max_pending = 0

    def push(self, samples):  # longform.rs:55-66
        self.pending.extend(samples)
        self.total += len(samples)
        self.max_pending = max(self.max_pending, len(self.pending))
        while self.next_block + self.block_samples + self.ctx_samples <= self.total:
            self.probs.extend(self._vad_block_at(self.next_block, self.next_block + self.block_samples))
            self.next_block += self.block_samples
        return self._drain(False)

    def flush(self):  # longform.rs:69-97, collect-only branch
        while self.next_block < self.total:
            end = min(self.next_block + self.block_samples, self.total)
            if end - self.next_block >= self.spf:
                self.probs.extend(self._vad_block_at(self.next_block, end))
            self.next_block = end
        return self._drain(True)

    def _vad_block_at(self, start, end):  # longform.rs:101-115
        lo = max(max(start - self.ctx_samples, 0), self.base_sample)
        lo = start - ((start - lo) // self.spf) * self.spf
        hi = min(end + self.ctx_samples, self.total)
        block = self.pending[lo - self.base_sample:hi - self.base_sample]
        return list(self.block_probs(block, (start - lo) // self.spf, (end - start) // self.spf))

    def _drain(self, fin):  # longform.rs:117-167
        out = []
        if not self.probs:
            if fin and len(self.pending) >= self.spf:
                out.append(self._emit(0, len(self.pending) // self.spf))
            return out
        segs = segment(self.probs, self.cfg)
        known = len(self.probs)
        closed = 0
        for i in range(len(segs)):
            is_closed = (fin or (i + 1 < len(segs) and segs[i + 1][1] + self.cfg["min_pause_frames"] <= known)
                         or (segs[i][1] - segs[i][0] >= self.cfg["max_frames"] and known >= segs[i][1] + 63))
            if not is_closed:
                break
            closed = i + 1
        if closed == 0:
            return out
        for s, e in segs[:closed]:
            out.append(self._emit(s, e))
        cut_frame = segs[closed][0] if closed < len(segs) else segs[closed - 1][1]
        cut_sample = min(cut_frame * self.spf, len(self.pending))
        del self.pending[:cut_sample]
        self.base_sample += cut_sample
        del self.probs[:min(cut_frame, len(self.probs))]
        return out

    def _emit(self, a, b):  # longform.rs:170-182, collect-only
        s0, s1 = a * self.spf, min(b * self.spf, len(self.pending))
        r = (self.base_sample + s0, self.base_sample + s1)
        self.ranges.append(r)
        return r
