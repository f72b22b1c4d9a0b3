"""Hugging Face route (transformers 5.5): MambaForCausalLM mixers on the B200 kernels.

CPU tests check the registration (the kernel-name mapping transformers consults when a mixer is
built, the modeling-module globals, and undoing both). GPU tests run a small random-init
MambaForCausalLM on CUDA through the patched fast path -- prefill (selective_scan_fn +
causal_conv1d_fn), training (mamba_inner_fn, with gradients) and cached decoding
(causal_conv1d_update + selective_state_update) -- against the same model on transformers' own
sequential PyTorch path.
"""

import contextlib

import pytest
import torch

transformers = pytest.importorskip("transformers")

from mamba_cpu_b200 import hf  # noqa: E402

from helpers import assert_close  # noqa: E402

FAST = ("causal_conv1d_fn", "causal_conv1d_update", "selective_state_update", "selective_scan_fn", "mamba_inner_fn")


def _config():
    from transformers import MambaConfig

    return MambaConfig(vocab_size=96, hidden_size=64, state_size=16, num_hidden_layers=2, expand=2, conv_kernel=4,
                       time_step_rank=8, use_mambapy=False)


@contextlib.contextmanager
def _patched():
    hf.patch_transformers()
    try:
        yield
    finally:
        hf.unpatch_transformers()


@contextlib.contextmanager
def _slow_path():
    """transformers' sequential PyTorch mixer: every fast-path function unset."""
    from transformers.models.mamba import modeling_mamba as mm

    saved = {n: getattr(mm, n, None) for n in FAST}
    for n in FAST:
        setattr(mm, n, None)
    try:
        yield
    finally:
        for n, v in saved.items():
            setattr(mm, n, v)


def test_patch_registers_modules_and_globals():
    from transformers.integrations import hub_kernels
    from transformers.models.mamba import modeling_mamba as mm

    before = dict(hub_kernels._KERNEL_MODULE_MAPPING)
    with _patched():
        mapping = hub_kernels._KERNEL_MODULE_MAPPING
        assert mapping["causal-conv1d"].causal_conv1d_fn is hf.causal_conv1d_fn
        assert mapping["causal-conv1d"].causal_conv1d_update is hf.causal_conv1d_update
        for n in ("selective_scan_fn", "selective_state_update", "mamba_inner_fn"):
            assert getattr(mapping["mamba-ssm"], n) is getattr(hf, n)
        # a mixer built now resolves the package's functions through lazy_load_kernel
        from transformers import MambaModel

        MambaModel(_config())
        for n in FAST:
            assert getattr(mm, n) is getattr(hf, n), n
    assert dict(hub_kernels._KERNEL_MODULE_MAPPING) == before


@pytest.mark.parametrize("family", ["falcon_mamba", "jamba"])
def test_patch_covers_other_families(family):
    """FalconMamba resolves through "falcon_mamba-ssm" and falcon_mamba_inner_fn; Jamba through
    "mamba-ssm" plus its cached is_fast_path_available flag. Both are undone by unpatching."""
    import importlib

    mod = importlib.import_module(f"transformers.models.{family}.modeling_{family}")
    names = ["causal_conv1d_fn", "causal_conv1d_update", "selective_state_update", "selective_scan_fn",
             "falcon_mamba_inner_fn" if family == "falcon_mamba" else "mamba_inner_fn"]
    if family == "jamba":
        names.append("is_fast_path_available")
    before = {n: getattr(mod, n, "<missing>") for n in names}
    with _patched():
        for n in names:
            want = True if n == "is_fast_path_available" else getattr(hf, n.replace("falcon_", ""))
            assert getattr(mod, n) is want, n
        if family == "falcon_mamba":
            from transformers import FalconMambaConfig, FalconMambaModel

            FalconMambaModel(FalconMambaConfig(vocab_size=32, hidden_size=16, state_size=4, num_hidden_layers=1))
            assert mod.falcon_mamba_inner_fn is hf.mamba_inner_fn
    assert {n: getattr(mod, n, "<missing>") for n in names} == before


def test_patch_covers_mamba2():
    """Mamba-2 resolves mamba_chunk_scan_combined / mamba_split_conv1d_scan_combined through
    "mamba-ssm"; a mixer built while patched reads the fast-path flag in forward, so unpatching
    leaves that flag False (transformers' own sequential path) rather than deleting it."""
    from transformers import Mamba2Config, Mamba2Model
    from transformers.models.mamba2 import modeling_mamba2 as m2

    names = ("causal_conv1d_fn", "causal_conv1d_update", "selective_state_update", "mamba_chunk_scan_combined",
             "mamba_split_conv1d_scan_combined")
    with _patched():
        Mamba2Model(Mamba2Config(vocab_size=32, hidden_size=64, state_size=16, num_heads=2, head_dim=64, expand=2,
                                 n_groups=1, num_hidden_layers=1))
        assert m2.is_fast_path_available is True
        assert m2.mamba_chunk_scan_combined is hf.ssd_chunk_scan
        assert m2.mamba_split_conv1d_scan_combined is hf.mamba_split_conv1d_scan_combined
        for n in names:
            assert getattr(m2, n) is not None, n
    assert m2.is_fast_path_available is False
    assert all(getattr(m2, n, None) is not hf.ssd_chunk_scan for n in names)


def test_mamba_inner_fn_signature_matches_mamba_ssm():
    import inspect

    params = list(inspect.signature(hf.mamba_inner_fn).parameters)
    assert params[:11] == ["xz", "conv1d_weight", "conv1d_bias", "x_proj_weight", "delta_proj_weight",
                           "out_proj_weight", "out_proj_bias", "A", "B", "C", "D"]
    for kw in ("delta_bias", "delta_softplus", "b_rms_weight", "c_rms_weight", "dt_rms_weight", "b_c_dt_rms_eps"):
        assert kw in params


@pytest.mark.parametrize("falcon", [False, True])
def test_mamba_inner_fn_composition(falcon, monkeypatch):
    """The composition around the ops (conv, projections, where the RMS norms sit, B/C projection
    biases) on CPU: hf.mamba_inner_fn with its two ops swapped for the plain-PyTorch references
    equals mamba_ssm's inner function restated in PyTorch, outputs and gradients."""
    from helpers import inner_fn_ref
    from mamba_cpu_b200 import causal_conv1d_ref, selective_scan_ref

    monkeypatch.setattr(hf, "causal_conv1d_fn", causal_conv1d_ref)
    monkeypatch.setattr(hf, "selective_scan_fn", selective_scan_ref)
    g = torch.Generator().manual_seed(5)
    b, d, r, n, L = 2, 12, 3, 4, 9

    def p(*shape, scale=0.5):
        return (torch.randn(*shape, generator=g, dtype=torch.float64) * scale).requires_grad_()

    args = [p(b, 2 * d, L), p(d, 1, 4), p(d), p(r + 2 * n, d), p(d, r), p(5, d), p(5),
            -torch.rand(d, n, generator=g, dtype=torch.float64).add(0.5).requires_grad_()]
    kw = dict(D=p(d), delta_bias=p(d, scale=0.1), delta_softplus=True)
    if falcon:
        kw.update(b_rms_weight=p(n), c_rms_weight=p(n), dt_rms_weight=p(d), b_c_dt_rms_eps=1e-6)
    else:
        kw.update(B_proj_bias=p(n), C_proj_bias=p(n))
    leaves = args + [v for v in kw.values() if isinstance(v, torch.Tensor)]
    outs = []
    for fn in (hf.mamba_inner_fn, inner_fn_ref):
        out = fn(*args, **kw)
        outs.append((out.detach(), torch.autograd.grad((out * out.detach().cos()).sum(), leaves)))
    # the two compositions associate the projections' float64 sums differently, and the reference
    # ops compute in float32 inside, so a last-bit difference can flip a float32 rounding
    torch.testing.assert_close(outs[0][0], outs[1][0], rtol=1e-6, atol=1e-8)
    for ga, gb in zip(outs[0][1], outs[1][1]):
        torch.testing.assert_close(ga, gb, rtol=1e-5, atol=1e-8)


def _model():
    from transformers import MambaForCausalLM

    torch.manual_seed(0)
    with _patched():
        model = MambaForCausalLM(_config())
    return model.cuda().float()


@pytest.mark.gpu
def test_prefill_matches_sequential_path():
    model = _model().eval()
    ids = torch.randint(0, 96, (2, 150), generator=torch.Generator().manual_seed(1)).cuda()
    with torch.no_grad(), _patched():
        fast = model(ids).logits
    with torch.no_grad(), _slow_path():
        ref = model(ids).logits
    assert_close(fast, ref, 1e-4, 1e-4, "logits")


@pytest.mark.gpu
def test_training_step_matches_sequential_path():
    model = _model().train()
    ids = torch.randint(0, 96, (2, 100), generator=torch.Generator().manual_seed(2)).cuda()
    with _patched():
        loss = model(ids, labels=ids).loss
        loss.backward()
    fast = {n: p.grad.detach().clone() for n, p in model.named_parameters() if p.grad is not None}
    fast_loss = loss.item()
    model.zero_grad(set_to_none=True)
    with _slow_path():
        loss = model(ids, labels=ids).loss
        loss.backward()
    assert abs(fast_loss - loss.item()) <= 1e-5 * abs(loss.item())
    assert len(fast) == sum(1 for _ in model.parameters())
    for n, p in model.named_parameters():
        scale = max(1e-6, float(p.grad.abs().max()))
        assert_close(fast[n] / scale, p.grad / scale, 1e-3, 1e-4, n)


@pytest.mark.gpu
def test_cached_decoding_matches_sequential_path():
    model = _model().eval()
    ids = torch.randint(0, 96, (2, 12), generator=torch.Generator().manual_seed(3)).cuda()
    kw = dict(max_new_tokens=6, do_sample=False, return_dict_in_generate=True, output_scores=True)
    with torch.no_grad(), _patched():
        fast = model.generate(ids, **kw)
    with torch.no_grad(), _slow_path():
        ref = model.generate(ids, **kw)
    assert torch.equal(fast.sequences, ref.sequences)
    for a, b in zip(fast.scores, ref.scores):
        assert_close(a, b, 1e-4, 1e-4, "scores")
