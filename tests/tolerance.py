"""bf16 comparison used by the GPU parity tests.

Two implementations that both round every op to bf16 (8 significant bits) can differ by one
rounding step anywhere upstream (a different GEMM summation order is enough), and such a step
moves a derived value by about 2^-8 of the magnitudes it was computed from, whatever its own
size; chained computations (the k-deep draft chain, 24 layers of verify) add such steps up.
So the bar "within 2e-2 in bf16" is checked two ways:

* every element within 2e-2 of the reference relative to the largest magnitude in the
  compared tensor (a logits tensor's largest logit, a state's largest entry);
* elementwise |got - want| <= 2e-2 + 2e-2 * |want| for all but 0.1 % of the elements (at least
  2 allowed): the usual elementwise bar on almost every value.
"""

import torch


def assert_bf16_close(got, want, tol=2e-2, outlier_frac=1e-3, what=""):
    g = got.detach().float().cpu()
    w = want.detach().float().cpu()
    assert g.shape == w.shape, (g.shape, w.shape)
    if g.numel() == 0:
        return
    d = (g - w).abs()
    scale = max(float(w.abs().max()), 1e-6)
    worst = float(d.max()) / scale
    assert worst <= tol, f"{what}: max |diff| / max |reference| = {worst:.4g} > {tol}"
    bad = int((d > tol + tol * w.abs()).sum())
    allowed = max(2, int(outlier_frac * d.numel()))
    assert bad <= allowed, f"{what}: {bad} of {d.numel()} elements beyond {tol} (atol and rtol); {allowed} allowed"


FP32_TOL = dict(rtol=1e-4, atol=1e-4)


def assert_close_dt(got, want, dt, what=""):
    """fp32: elementwise 1e-4 (relative and absolute); bf16: assert_bf16_close."""
    if dt == torch.bfloat16:
        assert_bf16_close(got, want, what=what)
    else:
        torch.testing.assert_close(got.detach().float().cpu(), want.detach().float().cpu(), **FP32_TOL)
