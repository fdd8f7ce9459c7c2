"""Numerical acceptance criteria for the krsi_b200 kernels.  TEST INFRASTRUCTURE ONLY.

`compare` restates the reference's judge (tools/common.py:322-392): a candidate passes when no
element is further from the fp32 result than `slack` x the original's worst element error
(+ 1e-3 x scale), its relative L2 error is within `slack` x the original's, and no row (flattened
over all but the last dim, rows of >= 64 elements) has a relative error above `row_slack` x the
original's error on the same row (floored at the median row error).  "Original" is the
reference's own eager path in the low-precision dtype.

`norm_max_err` is the BASELINE bound: max|c - r| / max|r| against the fp32 result (<= 1e-2 for
bf16 outputs and gradients); RMSNorm fp32 uses max-abs <= 1e-5 directly.
"""
from __future__ import annotations

import torch


def norm_max_err(cand: torch.Tensor, ref: torch.Tensor) -> float:
    r = ref.double()
    c = cand.double().to(r.device)
    scale = r.abs().max().item() or 1.0
    return (c - r).abs().max().item() / scale


def max_abs_err(cand: torch.Tensor, ref: torch.Tensor) -> float:
    return (cand.double().to(ref.device) - ref.double()).abs().max().item()


def compare(ref32, orig, cand, *, slack: float = 2.0, row_slack: float = 3.0) -> dict:
    """Lists of tensors in, {"pass": bool, "outputs": [per-tensor report]} out."""
    report, ok = [], True
    if len(ref32) != len(cand):
        return {"pass": False, "reason": f"output count {len(cand)} != {len(ref32)}"}
    for i, (r, o, c) in enumerate(zip(ref32, orig, cand)):
        item = {"output": i, "shape": list(r.shape)}
        if tuple(c.shape) != tuple(r.shape):
            item.update(passed=False, reason=f"shape {list(c.shape)} != {list(r.shape)}")
            report.append(item)
            ok = False
            continue
        r = r.float()
        o = o.float().to(r.device)
        c = c.float().to(r.device)
        scale = r.abs().max().item() or 1.0
        err_o, err_c = (o - r).abs(), (c - r).abs()
        budget = slack * err_o.max() + 1e-3 * scale + 1e-6
        bad = (err_c > budget) | ~torch.isfinite(c)
        rn_all = r.norm() + 1e-12
        rel_c = (err_c.norm() / rn_all).item()
        rel_o = (err_o.norm() / rn_all).item()
        passed = (not bad.any().item()) and rel_c <= slack * rel_o + 1e-5
        item.update(max_err=err_c.max().item(), orig_max_err=err_o.max().item(), rel_l2=rel_c,
                    orig_rel_l2=rel_o, bad_fraction=bad.float().mean().item())
        if r.dim() >= 2 and r.shape[-1] >= 64 and r.numel() // r.shape[-1] >= 2:
            r2 = r.reshape(-1, r.shape[-1])
            rown = r2.norm(dim=1)
            live = rown > 1e-6 * (rown.max() + 1e-30)
            if live.any():
                row_c = ((c - r).reshape(-1, r.shape[-1]).norm(dim=1) / (rown + 1e-30))[live]
                row_o = ((o - r).reshape(-1, r.shape[-1]).norm(dim=1) / (rown + 1e-30))[live]
                floor = row_o.median() + 1e-5
                bad_rows = int((row_c > row_slack * torch.maximum(row_o, floor)).sum())
                item["bad_rows"] = bad_rows
                passed = passed and bad_rows == 0
        item["passed"] = passed
        ok = ok and passed
        report.append(item)
    return {"pass": ok, "outputs": report}
