"""Small, profiler-friendly case of the benchmark workload.

    python -m flashmlp_b200.profile_case [--heads 4] [--rows 65536] [--act silu] [--iters 3]
                                         [--shared] [--allreduce]

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
    ap.add_argument("--dtype", default="bf16", choices=["bf16", "f16", "f32"])
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--only", choices=["fwd", "bwd", "both"], default="both")
    ap.add_argument("--shared", action="store_true",
                    help="shared-input kernels: one (B, D) input for all heads, head mean output")
    ap.add_argument("--fp8", action="store_true",
                    help="instead: the FP8 forward (flashmlp_fwd_fp8) on the e4m3-quantized inputs")
    ap.add_argument("--allreduce", action="store_true",
                    help="instead: fmlp_grad_allreduce_sgd (one rank) and fmlp_sgd_update on 2*H*D*E weights")
    a = ap.parse_args()
    dt = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}[a.dtype]
    H, B, D, E = a.heads, a.rows, a.hidden, a.inter
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(H, B, D, device="cuda", generator=g).to(dt)
    w1 = (torch.randn(H, D, E, device="cuda", generator=g) / D ** 0.5).to(dt)
    w2 = (torch.randn(H, E, D, device="cuda", generator=g) / E ** 0.5).to(dt)
    do = torch.randn(H, B, D, device="cuda", generator=g).to(dt)
    if a.allreduce:
        _allreduce(a, H, D, E, dt)
        return
    if a.fp8:
        from . import fp8
        x8, sx = fp8.quantize_e4m3(x)
        wq = fp8.prepare_fp8_weights(w1, w2)
        for _ in range(a.iters):
            fp8.flashmlp_fwd_fp8(x8, wq, a.act, x_scale=sx, h_scale=0.01)
        torch.cuda.synchronize()
        st = _lib.lib().fmlp_device_status(1)
        print(f"profile_case fp8 H={H} B={B} D={D} E={E} {a.act}: status {st}")
        if st:
            raise SystemExit(1)
        return
    if a.shared:
        x, do = x[0].contiguous(), do[0].contiguous()
    fwd = api.flashmlp_fwd_shared_x if a.shared else api.flashmlp_fwd
    bwd = api.flashmlp_bwd_shared_x if a.shared else api.flashmlp_bwd
    for _ in range(a.iters):
        if a.only in ("fwd", "both"):
            fwd(x, w1, w2, a.act)
        if a.only in ("bwd", "both"):
            bwd(x, w1, w2, do, a.act)
    torch.cuda.synchronize()
    st = _lib.lib().fmlp_device_status(1)
    print(f"profile_case H={H} B={B} D={D} E={E} {a.dtype} {a.act}: status {st}")
    if st:
        raise SystemExit(1)


def _allreduce(a, H, D, E, dt) -> None:
    """One-rank fmlp_grad_allreduce_sgd (barriers without peers; the reduce + update over all n
    weights) and fmlp_sgd_update, each `iters` times, on n = 2*H*D*E weights."""
    import ctypes

    n = 2 * H * D * E
    w = torch.randn(n, device="cuda").to(dt)
    g = torch.randn(n, device="cuda")
    flags = torch.zeros(_lib.FMLP_PEER_FLAG_WORDS, dtype=torch.int32, device="cuda")
    L = _lib.lib()
    arr = lambda t: (ctypes.c_void_p * 1)(ctypes.c_void_p(t.data_ptr()))
    code = _lib.FMLP_DTYPE_BF16 if dt == torch.bfloat16 else _lib.FMLP_DTYPE_F16
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for i in range(a.iters):
        rc = L.fmlp_grad_allreduce_sgd(arr(w), arr(g), arr(flags), 1, 0, n, 1e-4, code, 2 * i + 1, stream)
        _lib.check(rc, "fmlp_grad_allreduce_sgd")
        _lib.check(L.fmlp_sgd_update(ctypes.c_void_p(w.data_ptr()), ctypes.c_void_p(g.data_ptr()), n, 1e-4, code,
                                     stream), "fmlp_sgd_update")
    torch.cuda.synchronize()
    st = L.fmlp_device_status(1)
    print(f"profile_case allreduce n={n}: status {st}")
    if st:
        raise SystemExit(1)


if __name__ == "__main__":
    main()
