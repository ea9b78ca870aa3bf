"""Per-phase timeline of one decode step from the kernel's %globaltimer stamps.

The decode kernel writes, when tracing is enabled (mq_set_trace), one stamp per
CTA at the end of every phase of every layer.  `capture_step` runs one step with
tracing on and returns the stamps; `summarize` turns them into per-layer and
per-phase durations (max over CTAs, in microseconds).
"""
import statistics

import torch

from . import _lib

PHASES = ("start", "qkv", "attn", "oin", "o", "norm2", "gu", "mlpin", "down")
PER_LAYER = 10


def capture_step(decoder, token=5):
    """Runs one decode step of `decoder` with tracing; returns an int64 [num_ctas, slots] CPU tensor."""
    n = _lib.kernel_info()["num_ctas"]
    slots = PER_LAYER * (decoder.num_layers_ + 1)   # the last group: final hidden, LM head, entry, exit
    buf = torch.zeros(n, slots, dtype=torch.int64, device=decoder.device)
    _lib.set_trace(buf, slots)
    try:
        decoder.decode_steps(token, 1)
        torch.cuda.synchronize(decoder.device)
    finally:
        _lib.set_trace(None)
    return buf.cpu()


def summarize(stamps, num_layers):
    t = stamps.double()
    valid = t > 0
    t0 = t[:, 0][valid[:, 0]].min()
    rel = (t - t0) / 1000.0
    rel[~valid] = float("nan")

    def colmax(c):
        col = rel[:, c]
        col = col[~torch.isnan(col)]
        return float(col.max()) if len(col) else float("nan")

    layer = [colmax((l + 1) * PER_LAYER) - colmax(l * PER_LAYER) for l in range(num_layers - 1)]
    phase = {}
    for e in range(1, len(PHASES)):
        d = []
        for l in range(num_layers):
            a, b = colmax(l * PER_LAYER + e), colmax(l * PER_LAYER + e - 1)
            if a == a and b == b:
                d.append(a - b)
        if d:
            phase[PHASES[e]] = statistics.median(d)
    def colmin(c):
        col = rel[:, c]
        col = col[~torch.isnan(col)]
        return float(col.min()) if len(col) else float("nan")

    return {"layer_us_median": statistics.median(layer) if layer else None,
            "phase_us_median": phase,
            "kernel_entry_us": colmin(num_layers * PER_LAYER + 2),      # first CTA entered (negative: before layer 0)
            "final_hidden_us": colmax(num_layers * PER_LAYER),
            "lm_head_done_us": colmax(num_layers * PER_LAYER + 1),
            "kernel_done_us": colmax(num_layers * PER_LAYER + 3)}      # last CTA done
