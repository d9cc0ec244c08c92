"""Forward + backward on tensors that live in host memory, with the copies overlapped.

The reference's functions take device tensors (flashmlp.py:428-538); a caller whose data
sits in host memory first copies X, W1, W2 and dO to the GPU and the results back, and
those copies (2 x 16-bit x (2*H*B*D + 2*H*D*E) bytes per step) take longer than the
kernels over PCIe. Heads are independent, so `fwd_bwd_host` cuts the heads into groups
and pipelines them over three CUDA streams: group g+1 is copied in while group g runs
through flashmlp_fwd / flashmlp_bwd and group g-1 is copied out. Results are those of
flashmlp_fwd / flashmlp_bwd on each head group: O and dX are bit-identical to one call on
the whole tensors (the kernels treat heads independently); dW can differ from it in the
last bits, because a launch splits its dW sums over B ranges according to its head count
and the fp32 partials are then added in a different grouping.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from .api import flashmlp_bwd, flashmlp_fwd


def _pinned_like(t: torch.Tensor) -> torch.Tensor:
    return torch.empty(t.shape, dtype=t.dtype, pin_memory=True)


class HostPipeline:
    """Reusable device buffers and streams for `fwd_bwd_host` on one device.

    `heads_per_group` heads move and compute together; `slots` groups are in flight
    (3: one being copied in, one computing, one being copied out)."""

    def __init__(self, device=None, heads_per_group: int = 4, slots: int = 3, ramp: bool = True):
        dev = torch.device(device) if device is not None else torch.device("cuda")
        if dev.type != "cuda":
            raise RuntimeError("fwd_bwd_host computes on a CUDA device")
        self.device = dev if dev.index is not None else torch.device("cuda", torch.cuda.current_device())
        self.hg = max(1, int(heads_per_group))
        self.slots = max(2, int(slots))
        self.ramp = bool(ramp)
        self.s_in = torch.cuda.Stream(self.device)
        self.s_comp = torch.cuda.Stream(self.device)
        self.s_out = torch.cuda.Stream(self.device)
        self._key = None
        self._buf = None

    def _buffers(self, shapes, dtype):
        key = (shapes, dtype)
        if self._key != key:
            xs, w1s, w2s = shapes
            mk = lambda s: torch.empty(s, dtype=dtype, device=self.device)
            self._buf = [dict(x=mk(xs), w1=mk(w1s), w2=mk(w2s), do=mk(xs)) for _ in range(self.slots)]
            self._key = key
        return self._buf

    def _groups(self, H: int, hg: int):
        """Head ranges of the pipeline. With `ramp` (and room for it) the first and last
        groups are smaller (hg/4, hg/2, ..., hg/2, hg/4 heads), so that the copy-in before
        the first kernel and the copy-out after the last one are short."""
        if self.ramp and hg >= 2 and H >= 3 * hg:
            ends = sorted({max(1, hg // 4), max(1, hg // 2)})
            mid = H - 2 * sum(ends)
            sizes = ends + [hg] * (mid // hg) + ([mid % hg] if mid % hg else []) + ends[::-1]
        else:
            sizes = [min(hg, H - h0) for h0 in range(0, H, hg)]
        out, h0 = [], 0
        for n in sizes:
            out.append((h0, h0 + n))
            h0 += n
        assert h0 == H
        return out

    def run(self, x: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor, do: torch.Tensor, activation: str = "",
            out: Optional[Tuple[torch.Tensor, ...]] = None):
        """x, do (H, B, D), w1 (H, D, E), w2 (H, E, D) in (preferably pinned) host memory.
        Returns host tensors (o, dx, dw1, dw2), written into `out` when given."""
        H, B, D = x.shape
        E = w1.shape[2]
        if out is None:
            out = (_pinned_like(x), _pinned_like(x), _pinned_like(w1), _pinned_like(w2))
        o_h, dx_h, dw1_h, dw2_h = out
        hg = min(self.hg, max(H, 1))
        bufs = self._buffers(((hg, B, D), (hg, D, E), (hg, E, D)), x.dtype)
        groups = self._groups(H, hg)
        # Per group, the forward needs only X, W1, W2 and its output O can go back while the
        # backward runs, so the copies are split: X, W1, W2 in -> forward -> (O out | dO in)
        # -> backward -> dX, dW1, dW2 out. The pipeline's fill (before the first kernel) and
        # drain (after the last) then carry about half the bytes of a group each way.
        ev_xw = [torch.cuda.Event() for _ in groups]
        ev_do = [torch.cuda.Event() for _ in groups]
        ev_fwd = [torch.cuda.Event() for _ in groups]
        ev_comp = [torch.cuda.Event() for _ in groups]
        ev_out = [torch.cuda.Event() for _ in groups]
        # the slots may still be read by the previous call's work, and the caller's stream
        # may have queued work this call must follow
        self.s_in.wait_stream(self.s_out)
        self.s_in.wait_stream(torch.cuda.current_stream(self.device))
        for g, (a, b) in enumerate(groups):
            n = b - a
            slot = bufs[g % self.slots]
            if g >= self.slots:  # the slot's previous group has been copied out
                self.s_in.wait_event(ev_out[g - self.slots])
            with torch.cuda.stream(self.s_in):
                for k, src in (("x", x), ("w1", w1), ("w2", w2)):
                    slot[k][:n].copy_(src[a:b], non_blocking=True)
                ev_xw[g].record(self.s_in)
                slot["do"][:n].copy_(do[a:b], non_blocking=True)
                ev_do[g].record(self.s_in)
            xs, w1s, w2s, dos = (slot[k][:n] for k in ("x", "w1", "w2", "do"))
            self.s_comp.wait_event(ev_xw[g])
            with torch.cuda.stream(self.s_comp):
                o = flashmlp_fwd(xs, w1s, w2s, activation)
                ev_fwd[g].record(self.s_comp)
            self.s_out.wait_event(ev_fwd[g])
            with torch.cuda.stream(self.s_out):
                o_h[a:b].copy_(o, non_blocking=True)
                o.record_stream(self.s_out)
            self.s_comp.wait_event(ev_do[g])
            with torch.cuda.stream(self.s_comp):
                grads = flashmlp_bwd(xs, w1s, w2s, dos, activation)
                ev_comp[g].record(self.s_comp)
            self.s_out.wait_event(ev_comp[g])
            with torch.cuda.stream(self.s_out):
                for dst, src in zip((dx_h, dw1_h, dw2_h), grads):
                    dst[a:b].copy_(src, non_blocking=True)
                    src.record_stream(self.s_out)
                ev_out[g].record(self.s_out)
            del o, grads
        torch.cuda.current_stream(self.device).wait_stream(self.s_out)
        return o_h, dx_h, dw1_h, dw2_h


def fwd_bwd_host(x: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor, do: torch.Tensor, activation: str = "",
                 device=None, heads_per_group: int = 4):
    """One forward + backward of host-resident tensors on `device` (default: the current
    CUDA device), copies overlapped with the kernels. Returns host (o, dx, dw1, dw2); the
    host outputs are complete once torch.cuda.current_stream() has synchronised."""
    return HostPipeline(device, heads_per_group).run(x, w1, w2, do, activation)
