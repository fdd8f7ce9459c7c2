"""Run one small case of a krsi_b200 kernel (for profilers such as ncu): three warm-up calls and
one more, on seeded inputs.

  python kernel-rsi_b200/profile_case.py rmsnorm|rmsnorm_bf16|geglu|attn_fwd|attn ROWS_OR_B [S]

rmsnorm / rmsnorm_bf16: x [ROWS, 1152] fp32 / bf16 fwd+bwd; geglu: u [ROWS, 9216] bf16 fwd+bwd;
attn_fwd / attn: relpos attention B=ROWS_OR_B, S, H=16, D=72 bf16 (fwd / fwd+bwd).
"""
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))
sys.path.insert(0, str(HERE / "library"))
import _ext  # noqa: E402  (loads the native libraries)


def gen(shape, seed, dtype, std=1.0, mean=0.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(shape, generator=g) * std + mean).to(dtype).cuda()


def main():
    which = sys.argv[1]
    n = int(sys.argv[2])
    ops = torch.ops.krsi
    for _ in range(4):
        if which in ("rmsnorm", "rmsnorm_bf16"):
            dt = torch.float32 if which == "rmsnorm" else torch.bfloat16
            x, g = gen((n, 1152), 0, dt), gen((n, 1152), 2, dt)
            w = gen((1152,), 1, dt, 0.02, 1.0)
            y, r = ops.rmsnorm_fwd(x, w, 1e-6)
            ops.rmsnorm_bwd(g, x, w, r)
        elif which == "geglu":
            u, g = gen((n, 9216), 0, torch.bfloat16), gen((n, 4608), 1, torch.bfloat16)
            ops.geglu_fwd(u)
            ops.geglu_bwd(g, u)
        else:
            S, H, D = int(sys.argv[3]), 16, 72
            qkv = gen((n * S, 3 * H * D), 0, torch.bfloat16, D ** -0.5)
            pd = gen((H, 2 * S - 1), 1, torch.float32, 0.02)
            out, out32, lse = ops.relpos_attn_fwd(qkv, pd, n, S, H, D, D ** -0.5)
            if which == "attn":
                dout = gen((n * S, H * D), 2, torch.bfloat16)
                ops.relpos_attn_bwd(dout, qkv, pd, out32, lse, n, S, H, D, D ** -0.5)
    torch.cuda.synchronize()
    assert _ext.device_status(clear=True) == 0
    print("ok", which)


if __name__ == "__main__":
    main()
