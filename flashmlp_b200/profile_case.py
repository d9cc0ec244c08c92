"""Small, profiler-friendly case of the benchmark workload.

    python -m flashmlp_b200.profile_case [--heads 4] [--rows 65536] [--act silu] [--iters 3]

Runs `iters` forward and `iters` backward launches of the C4 shape restricted to a few
heads (inputs still larger than L2), so an ncu capture of one launch stays small:
    ncu --set full --clock-control none -k regex:fmlp_bwd -s 1 -c 1 -o prof \
        python -m flashmlp_b200.profile_case
"""
from __future__ import annotations

import argparse

import torch

from . import api, _lib


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--heads", type=int, default=4)
    ap.add_argument("--rows", type=int, default=65536)
    ap.add_argument("--hidden", type=int, default=128)
    ap.add_argument("--inter", type=int, default=2048)
    ap.add_argument("--act", default="silu")
    ap.add_argument("--dtype", default="bf16", choices=["bf16", "f16"])
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--only", choices=["fwd", "bwd", "both"], default="both")
    a = ap.parse_args()
    dt = torch.bfloat16 if a.dtype == "bf16" else torch.float16
    H, B, D, E = a.heads, a.rows, a.hidden, a.inter
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(H, B, D, device="cuda", generator=g).to(dt)
    w1 = (torch.randn(H, D, E, device="cuda", generator=g) / D ** 0.5).to(dt)
    w2 = (torch.randn(H, E, D, device="cuda", generator=g) / E ** 0.5).to(dt)
    do = torch.randn(H, B, D, device="cuda", generator=g).to(dt)
    for _ in range(a.iters):
        if a.only in ("fwd", "both"):
            api.flashmlp_fwd(x, w1, w2, a.act)
        if a.only in ("bwd", "both"):
            api.flashmlp_bwd(x, w1, w2, do, a.act)
    torch.cuda.synchronize()
    st = _lib.lib().fmlp_device_status(1)
    print(f"profile_case H={H} B={B} D={D} E={E} {a.dtype} {a.act}: status {st}")
    if st:
        raise SystemExit(1)


if __name__ == "__main__":
    main()
