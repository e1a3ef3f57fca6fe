"""NEED's model forward with every recurrent layer routed through the drop-in.

The reference model (need_core.NeedModel, need_core.py:3984-4230) imports the
kernel module by name (need_core.py:33-36) and calls it at run time: with the
preset's retention_impl="ssd", StructuredDualRetention's ssd_scan under no_grad
(need_core.py:1624-1629), once per layer, plus rms_norm and swiglu.  (The
reference's own ssd_scan runs its torch path through affine_recurrence_scan,
need_kernels.py:336-337; the drop-in's ssd_scan is one kernel.)  This test builds the
~350M preset of config_for_size.model_config_for_params (d_model=832, 14
layers, block_size raised to 2048 for 2048-token rows), seeded N(0, 0.02)
weights from the model's own _init_weights, eval, and runs one forward over an
8 x 2048 batch of token ids ~ U[0, vocab) in bf16 the way the reference runs
inference (fp32 weights under torch.autocast(dtype=bfloat16), generate.py:1334),
so the scans see bf16 streams, twice:

* with the reference's own need_kernels on its torch path (Triton off: the
  path whose rounding points the CUDA kernels follow), and
* with need_b200.need_kernels bound in its place,

and requires all 14 ssd_scan calls to go through libneed_scan.so, each call's
output to agree with the reference's torch-path ssd_scan on that call's own
inputs within the bf16 budget (max |diff| / max |ref| <= 2e-2), and the logits,
where the 14 layers compound the gates' last-bit roundings, to agree within
the same budget.  The reference's Triton path (fp32 gate math) is run as well
and its distance reported.  The reference model takes no reset mask, so no
arm uses resets.  Both arms run with the config's image_2d_scan off: that
module calls affine_recurrence_scan_torch directly (need_core.py:1769), not the
kernel module, and under CUDA autocast it writes its bf16 result into a float32
buffer (need_core.py:1779, :1820) and raises once a random image span is long
enough to form a grid.

The reference is imported from baseline/_ref (an unmodified copy made by
baseline/fetch_reference.sh, git-ignored); without it the test is skipped.
"""
import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")

pytestmark = pytest.mark.gpu

BF16_TOL = 2e-2
B, T = 8, 2048


def reference_modules():
    if not os.path.exists(os.path.join(REF, "need_core.py")):
        pytest.skip("baseline/_ref has no copy of the reference (run baseline/fetch_reference.sh)")
    sys.dont_write_bytecode = True
    if REF not in sys.path:
        sys.path.insert(0, REF)
    import config_for_size  # noqa: E402
    import need_core  # noqa: E402
    import need_kernels  # noqa: E402  (the reference's module of that name)
    return need_core, need_kernels, config_for_size


def build_model(need_core, config_for_size, dev, **overrides):
    cfg, _ = config_for_size.model_config_for_params(350_000_000, block_size=T)
    cfg["image_2d_scan"] = False
    cfg.update(overrides)
    torch.manual_seed(0)
    with torch.device(dev):
        model = need_core.NeedModel(need_core.NeedConfig(**cfg))
    return model.eval(), cfg


def forward_logits(model, ids):
    with torch.no_grad(), torch.autocast(device_type="cuda", dtype=torch.bfloat16):
        out = model(ids)
    torch.cuda.synchronize()
    return out[0].float()


def rel(a, b):
    return float((a - b).abs().max() / b.abs().max()), float((a - b).norm() / b.norm())


def test_need_model_forward_through_the_drop_in(cuda):
    need_core, ref_nk, config_for_size = reference_modules()
    from need_b200 import need_kernels as nk

    model, cfg = build_model(need_core, config_for_size, cuda)
    assert (cfg["d_model"], cfg["n_layers"]) == (832, 14)
    gen = torch.Generator(device=cuda).manual_seed(5)
    ids = torch.randint(0, model.cfg.vocab_size, (B, T), device=cuda, generator=gen)

    saved_binding, saved_triton = need_core.need_kernels, ref_nk.HAS_TRITON
    try:
        # the reference's torch path
        need_core.need_kernels = ref_nk
        ref_nk.HAS_TRITON = False
        want = forward_logits(model, ids)
        # the reference's Triton path (informational)
        ref_nk.HAS_TRITON = saved_triton
        triton_logits = forward_logits(model, ids) if saved_triton else None

        # the drop-in, counting the scan calls that reach the library and
        # keeping each ssd_scan call's inputs and output
        calls = {"ssd_scan": 0, "affine_recurrence_scan": 0}
        recorded = []

        class Counting:
            def __getattr__(self, name):
                fn = getattr(nk, name)
                if name not in calls:
                    return fn

                def counted(*a, **k):
                    calls[name] += 1
                    y = fn(*a, **k)
                    if name == "ssd_scan":
                        recorded.append(([t.clone() if isinstance(t, torch.Tensor) else t for t in a], y.clone()))
                    return y
                return counted

        need_core.need_kernels = Counting()
        got = forward_logits(model, ids)
    finally:
        need_core.need_kernels = saved_binding
        ref_nk.HAS_TRITON = saved_triton

    assert calls == {"ssd_scan": 14, "affine_recurrence_scan": 0}, calls
    assert nk.workspace_error() == 0
    # every layer's scan against the reference's torch path on the same inputs
    ref_nk.HAS_TRITON = False
    try:
        worst = 0.0
        for i, (args, y) in enumerate(recorded):
            with torch.no_grad():
                want_y = ref_nk.ssd_scan(*args)
            e, _ = rel(y.float(), want_y.float())
            worst = max(worst, e)
            assert e <= BF16_TOL, f"layer {i}: ssd_scan max rel {e}"
    finally:
        ref_nk.HAS_TRITON = saved_triton
    print(f"\nper-layer ssd_scan vs the reference's torch path: worst max rel {worst:.3e}")
    assert torch.isfinite(got).all()
    err, l2 = rel(got, want)
    print(f"\nlogits vs the reference's torch path: max rel {err:.3e}, rel L2 {l2:.3e}")
    if triton_logits is not None:
        terr, tl2 = rel(got, triton_logits)
        rerr, rl2 = rel(want, triton_logits)
        print(f"logits vs the reference's Triton path: max rel {terr:.3e}, rel L2 {tl2:.3e} "
              f"(the reference's own torch path vs its Triton path: {rerr:.3e}, {rl2:.3e})")
    assert err <= BF16_TOL, f"logits differ from the reference's: max rel {err}"


def test_ssd_block_patched_with_the_folded_conv(cuda):
    """The maintainer's patch: StructuredDualRetention.forward under no_grad as
    in_proj -> ssd_conv_scan (the conv + SiLU folded into the scan, then the
    out_norm kernel) -> out, with need_b200.need_kernels bound for the rest
    of the model.  Every one of the 14 blocks is compared with the reference's
    own block forward (torch path) on the input the reference's forward gave
    it, within the bf16 budget; then the whole forward runs with the patch."""
    need_core, ref_nk, config_for_size = reference_modules()
    from need_b200 import need_kernels as nk

    model, _ = build_model(need_core, config_for_size, cuda)
    gen = torch.Generator(device=cuda).manual_seed(6)
    ids = torch.randint(0, model.cfg.vocab_size, (B, T), device=cuda, generator=gen)
    SDR = need_core.StructuredDualRetention
    original = SDR.forward

    def patched(self, x):
        if torch.is_grad_enabled():
            return original(self, x)
        u, bg, cg, dt, og = self.in_proj(x).chunk(5, dim=-1)
        y = nk.ssd_conv_scan(u, bg, cg, dt, og, self.D, self.cfg.ssd_dt_min, self.cfg.ssd_dt_max,
                             self.dwconv.weight, self.dwconv.bias,
                             norm_weight=self.out_norm.weight, eps=self.out_norm.eps)
        return self.out(y)

    blocks = [m for m in model.modules() if isinstance(m, SDR)]
    assert len(blocks) == 14
    seen = []
    hooks = [m.register_forward_pre_hook(lambda m, a: seen.append((m, a[0].detach().clone()))) for m in blocks]
    saved_binding, saved_triton = need_core.need_kernels, ref_nk.HAS_TRITON
    try:
        need_core.need_kernels = ref_nk
        ref_nk.HAS_TRITON = False
        want = forward_logits(model, ids)
        for h in hooks:
            h.remove()
        worst = 0.0
        for i, (m, x) in enumerate(seen):
            with torch.no_grad(), torch.autocast(device_type="cuda", dtype=torch.bfloat16):
                ref_y = original(m, x)
                need_core.need_kernels = nk
                got_y = patched(m, x)
                need_core.need_kernels = ref_nk
            e, _ = rel(got_y.float(), ref_y.float())
            worst = max(worst, e)
            assert e <= BF16_TOL, f"block {i}: max rel {e}"
        need_core.need_kernels = nk
        SDR.forward = patched
        got = forward_logits(model, ids)
    finally:
        SDR.forward = original
        need_core.need_kernels = saved_binding
        ref_nk.HAS_TRITON = saved_triton
    assert nk.workspace_error() == 0
    assert torch.isfinite(got).all()
    err, l2 = rel(got, want)
    print(f"\nper-block (patched vs the reference's block): worst max rel {worst:.3e}; "
          f"logits: max rel {err:.3e}, rel L2 {l2:.3e}")
    assert err <= BF16_TOL, f"logits differ from the reference's: max rel {err}"


def test_need_model_training_step_through_the_drop_in(cuda):
    """NEED's training path: with gradients on, every StructuredDualRetention
    block computes its gates as torch ops and calls
    need_kernels.affine_recurrence_scan under autograd (need_core.py:1630-1638),
    whose backward here is the reversed-time scan kernel.

    The reference arm runs that scan as the reference's own differentiable
    chunked torch scan (_chunked_affine_recurrence_scan, need_kernels.py:
    177-226: its CPU path, and its CUDA path when associative_scan is
    missing), not its CUDA associative_scan route (:245-262): on this torch
    that route returns the right states and update gradient but loses the
    decay gradient (relative error 1.0 against float64 autograd at
    2 x 1024 x 832, where the chunked scan and this library's kernel are
    within 3e-3).  Everything else comes from the reference.  One forward, a
    cross-entropy of the logits against targets ~ U[0, vocab) (the model's own
    loss path calls binary_cross_entropy, which torch refuses under autocast),
    and the backward over 2 x 1024 tokens, in training mode with the preset's
    dropout set to 0 (the model's cuDNN RNN runs backward only in training
    mode; no other module draws random numbers at these settings), bf16
    autocast, with the reference's need_kernels (torch path) and with the
    drop-in.  All 14 forward scans and 14 adjoint
    scans must run in libneed_scan.so; the loss must agree to 1e-3 relative,
    the whole gradient (every parameter, one vector) within 2e-2 relative L2,
    and the gradient of every parameter of the 14 SSD blocks within 5e-2
    relative L2 (bf16 roundings of the gates compound through 14 layers and
    the backward).  Parameters elsewhere are checked only through the whole
    vector: some get gradients near zero, where a relative error says
    nothing."""
    need_core, ref_nk, config_for_size = reference_modules()
    from need_b200 import need_kernels as nk

    model, _ = build_model(need_core, config_for_size, cuda, dropout=0.0)
    model.train()
    gen = torch.Generator(device=cuda).manual_seed(7)
    bt, tt = 2, 1024
    ids = torch.randint(0, model.cfg.vocab_size, (bt, tt), device=cuda, generator=gen)
    targets = torch.randint(0, model.cfg.vocab_size, (bt, tt), device=cuda, generator=gen)

    def step(binding):
        need_core.need_kernels = binding
        model.zero_grad(set_to_none=True)
        with torch.enable_grad(), torch.autocast(device_type="cuda", dtype=torch.bfloat16):
            logits = model(ids)[0]
        loss = torch.nn.functional.cross_entropy(logits.float().reshape(-1, logits.shape[-1]), targets.reshape(-1))
        loss.backward()
        torch.cuda.synchronize()
        return float(loss.detach()), {n: p.grad.float().clone() for n, p in model.named_parameters()
                                      if p.grad is not None}

    calls = {"forward": 0, "adjoint": 0}
    adjoint = nk._affine_adjoint

    def counted_adjoint(*a, **k):
        calls["adjoint"] += 1
        return adjoint(*a, **k)

    class Counting:
        def __getattr__(self, name):
            fn = getattr(nk, name)
            if name != "affine_recurrence_scan":
                return fn

            def counted(*a, **k):
                calls["forward"] += 1
                return fn(*a, **k)
            return counted

    class ReferenceChunked:
        """The reference's module with its differentiable chunked scan."""

        def __getattr__(self, name):
            if name == "affine_recurrence_scan":
                return lambda decay, update, *, dim=1, backend="auto": ref_nk._chunked_affine_recurrence_scan(
                    torch.broadcast_to(decay, update.shape), update, dim=dim)
            return getattr(ref_nk, name)

    saved_binding, saved_triton = need_core.need_kernels, ref_nk.HAS_TRITON
    try:
        ref_nk.HAS_TRITON = False
        want_loss, want = step(ReferenceChunked())
        nk._affine_adjoint = counted_adjoint
        got_loss, got = step(Counting())
    finally:
        nk._affine_adjoint = adjoint
        need_core.need_kernels = saved_binding
        ref_nk.HAS_TRITON = saved_triton
    assert calls == {"forward": 14, "adjoint": 14}, calls
    assert nk.workspace_error() == 0
    assert set(got) == set(want)
    lerr = abs(got_loss - want_loss) / abs(want_loss)
    names = sorted(got)
    gv = torch.cat([got[n].flatten() for n in names])
    wv = torch.cat([want[n].flatten() for n in names])
    gerr = float((gv - wv).norm() / wv.norm())
    ssd = tuple(name + "." for name, m in model.named_modules() if isinstance(m, need_core.StructuredDualRetention))
    assert len(ssd) == 14
    worst, worst_name, nssd = 0.0, "", 0
    for name in names:
        if not name.startswith(ssd):
            continue
        nssd += 1
        e = float((got[name] - want[name]).norm() / want[name].norm().clamp_min(1e-30))
        if e > worst:
            worst, worst_name = e, name
    print(f"\nloss {got_loss:.6f} vs {want_loss:.6f} (rel {lerr:.2e}); whole gradient rel L2 {gerr:.3e} "
          f"over {len(names)} tensors; worst of the {nssd} SSD-block tensors {worst:.3e} ({worst_name})")
    assert lerr <= 1e-3
    assert gerr <= 2e-2
    assert worst <= 5e-2, worst_name
