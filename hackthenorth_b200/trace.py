"""Per-launch timeline of one captured decode step, from the kernels' own
``%globaltimer`` stamps (``qb_set_trace`` in ``include/qb.h``).

Every CTA of a traced launch records its start, the return of
``griddepcontrol.wait``, the landing of its first input stage, the end of its
main loop and its exit. ``StepTrace.summary`` turns that into, per launch, how
far the step advanced while it was the last to finish (``span``, summing to the
step time), how long after its predecessor's last CTA ended its waits returned
(``release``), and when its CTAs started relative to that predecessor's end.
This is how the time between kernels of a pipelined step (programmatic
dependent launch inside a CUDA graph) is apportioned, which a serialising
profiler cannot show. Diagnostics only: a traced step runs the same kernels
with a few extra global stores per CTA.
"""
from __future__ import annotations

import statistics
from typing import Dict, List

import torch

from . import _lib

MAX_CTAS = 256
STAMPS = 8
ENTRY, WAIT, FIRST, LOOP, EXIT, MERGED, CWAIT, CSYNC = range(8)


class StepTrace:
    """Trace records for up to ``max_launches`` launches of ``state``'s step.
    Call before the state captures its graph (it drops a captured graph)."""

    def __init__(self, state, max_launches: int = 512):
        self.state = state
        self.engine = state.engine
        self.max_launches = max_launches
        self.buf = torch.zeros(max_launches * MAX_CTAS * STAMPS, dtype=torch.int64, device=state.token.device)
        _lib.check(_lib.load().qb_set_trace(self.engine.ctx, self.buf.data_ptr(),
                                            self.buf.numel() * self.buf.element_size()), self.engine.ctx)
        state.captured = False

    def close(self) -> None:
        _lib.check(_lib.load().qb_set_trace(self.engine.ctx, None, 0), self.engine.ctx)
        self.state.captured = False

    def labels(self) -> List[str]:
        raw = _lib.load().qb_trace_labels(self.engine.ctx).decode()
        return [x for x in raw.split("\n") if x]

    def launches(self) -> List[Dict]:
        """Raw per-launch records of the latest traced step: label and, per
        recorded CTA, its stamps in ns (0 = not taken)."""
        labels = self.labels()
        recs = self.buf.view(self.max_launches, MAX_CTAS, STAMPS)[:len(labels)].cpu()
        out = []
        for i, name in enumerate(labels):
            r = recs[i]
            r = r[r[:, ENTRY] > 0]
            out.append({"label": name, "stamps": r})
        return out

    def summary(self) -> Dict:
        """Per launch (times in µs): ``start`` of its first CTA and ``end`` of its
        last CTA relative to the step's first CTA start; ``span`` = end minus the
        previous launch's end; ``release`` = its last griddepcontrol.wait return
        minus the previous launch's end; ``first`` = median time from a CTA's
        start to its first landed input stage; ``ctas``. Plus per-kind sums of
        span and release over the step."""
        rows = self.launches()
        if not rows:
            return {"launches": [], "step_us": 0.0}
        t0 = min(int(r["stamps"][:, ENTRY].min()) for r in rows if len(r["stamps"]))
        out, prev_end = [], None
        kinds: Dict[str, Dict[str, float]] = {}
        for r in rows:
            s = r["stamps"]
            if len(s) == 0:
                continue
            start = (int(s[:, ENTRY].min()) - t0) / 1e3
            end = (int(s[:, EXIT].max()) - t0) / 1e3
            waits = s[:, WAIT][s[:, WAIT] > 0]
            wait = (int(waits.max()) - t0) / 1e3 if len(waits) else None
            firsts = [(int(a) - int(b)) / 1e3 for a, b in zip(s[:, FIRST], s[:, ENTRY]) if int(a) > 0]
            rec = {"label": r["label"], "ctas": int(len(s)), "start": round(start, 2), "end": round(end, 2),
                   "span": round(end - (prev_end if prev_end is not None else start), 2),
                   "release": None if (wait is None or prev_end is None) else round(wait - prev_end, 2),
                   "first": round(statistics.median(firsts), 2) if firsts else None}
            # per CTA, each stamp relative to the CTA's start: median and max
            for k, name in ((WAIT, "wait"), (FIRST, "first"), (LOOP, "loop"), (MERGED, "merged"),
                            (CWAIT, "cwait"), (CSYNC, "csync"), (EXIT, "exit")):
                offs = [(int(a) - int(b)) / 1e3 for a, b in zip(s[:, k], s[:, ENTRY]) if int(a) > 0]
                if offs:
                    rec[f"{name}_med"] = round(statistics.median(offs), 2)
                    rec[f"{name}_max"] = round(max(offs), 2)
            out.append(rec)
            kind = r["label"].split()[0]
            k = kinds.setdefault(kind, {"launches": 0, "span_us": 0.0, "release_us": 0.0})
            k["launches"] += 1
            k["span_us"] = round(k["span_us"] + rec["span"], 2)
            if rec["release"] is not None:
                k["release_us"] = round(k["release_us"] + rec["release"], 2)
            prev_end = end
        return {"step_us": round(out[-1]["end"] - out[0]["start"], 2), "by_kind": kinds, "launches": out}
