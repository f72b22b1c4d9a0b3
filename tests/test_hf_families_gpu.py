"""The Hugging Face route for the other Mamba-1 families transformers 5.5 ships: FalconMamba and
Jamba, plus padded batches (an attention mask with left padding) for all three families.

mamba-cpu tests its route on Mamba, FalconMamba and Jamba (tests/test_hf.py:15-30) and on a padded
batch (:92-104). Here each small random-init model runs on CUDA through the patched fast path --
FalconMamba's training step goes through ``falcon_mamba_inner_fn`` with its RMS-normalised dt, B
and C; Jamba's mixer calls ``selective_scan_fn`` and ``causal_conv1d_fn`` itself -- and is compared
with the same model on transformers' own sequential PyTorch mixer.
"""

import contextlib
import importlib

import pytest
import torch

transformers = pytest.importorskip("transformers")

from mamba_cpu_b200 import hf  # noqa: E402

from helpers import assert_close, inner_fn_ref  # noqa: E402

pytestmark = pytest.mark.gpu

FAMILIES = ("mamba", "falcon_mamba", "jamba")
_FAST = {
    "mamba": ("causal_conv1d_fn", "causal_conv1d_update", "selective_state_update", "selective_scan_fn",
              "mamba_inner_fn"),
    "falcon_mamba": ("causal_conv1d_fn", "causal_conv1d_update", "selective_state_update", "selective_scan_fn",
                     "falcon_mamba_inner_fn"),
}


def _build(family):
    torch.manual_seed(0)
    if family == "mamba":
        cfg = transformers.MambaConfig(vocab_size=80, hidden_size=48, state_size=16, num_hidden_layers=2, expand=2,
                                       conv_kernel=4, time_step_rank=6, use_mambapy=False)
        cls = transformers.MambaForCausalLM
    elif family == "falcon_mamba":
        cfg = transformers.FalconMambaConfig(vocab_size=80, hidden_size=48, state_size=16, num_hidden_layers=2,
                                             expand=2, conv_kernel=4, time_step_rank=6, use_mambapy=False)
        cls = transformers.FalconMambaForCausalLM
    else:
        cfg = transformers.JambaConfig(vocab_size=80, hidden_size=48, intermediate_size=96, num_hidden_layers=2,
                                       num_attention_heads=4, num_key_value_heads=2, num_experts=1,
                                       attn_layer_period=2, attn_layer_offset=1, expert_layer_period=2,
                                       expert_layer_offset=1, mamba_d_state=16, mamba_dt_rank=6,
                                       mamba_expand=2, use_mamba_kernels=True)
        cls = transformers.JambaForCausalLM
    hf.patch_transformers()  # the mixers resolve their kernels when they are built
    try:
        model = cls(cfg)
    finally:
        hf.unpatch_transformers()
    return model.cuda().float()


@contextlib.contextmanager
def _fast(model, family):
    hf.patch_transformers()
    try:
        yield
    finally:
        hf.unpatch_transformers()


@contextlib.contextmanager
def _slow(model, family):
    """transformers' sequential mixer: Mamba / FalconMamba with their fast-path functions unset,
    Jamba with use_mamba_kernels off."""
    if family == "jamba":
        saved = model.config.use_mamba_kernels
        model.config.use_mamba_kernels = False
        try:
            yield
        finally:
            model.config.use_mamba_kernels = saved
        return
    mod = importlib.import_module(f"transformers.models.{family}.modeling_{family}")
    saved = {n: getattr(mod, n, None) for n in _FAST[family]}
    for n in saved:
        setattr(mod, n, None)
    try:
        yield
    finally:
        for n, v in saved.items():
            setattr(mod, n, v)


def _scan_calls(monkeypatch):
    """Counts the package's selective-scan calls through the patched route."""
    import mamba_cpu_b200.ops.selective_scan_interface as ssi

    calls = []
    real = ssi.selective_scan_fn

    def counting(*a, **k):
        calls.append(1)
        return real(*a, **k)

    monkeypatch.setattr(hf, "selective_scan_fn", counting)
    return calls


@pytest.mark.parametrize("family", ["falcon_mamba", "jamba"])
def test_prefill_matches_sequential_path(family, monkeypatch):
    model = _build(family).eval()
    ids = torch.randint(0, 80, (2, 70), generator=torch.Generator().manual_seed(1)).cuda()
    calls = _scan_calls(monkeypatch)
    with torch.no_grad(), _fast(model, family):
        fast = model(ids).logits
    assert calls, "the patched selective scan was not used"
    with torch.no_grad(), _slow(model, family):
        ref = model(ids).logits
    assert_close(fast, ref, 1e-4, 1e-4, "logits")


def _grads(model, ids):
    model.zero_grad(set_to_none=True)
    loss = model(ids, labels=ids).loss
    loss.backward()
    return loss.item(), {n: p.grad.detach().clone() for n, p in model.named_parameters() if p.grad is not None}


def _compare_grads(fast, ref):
    (fl, fg), (rl, rg) = fast, ref
    assert abs(fl - rl) <= 1e-5 * abs(rl)
    assert fg.keys() == rg.keys()
    for n in rg:
        scale = max(1e-6, float(rg[n].abs().max()))
        assert_close(fg[n] / scale, rg[n] / scale, 1e-3, 1e-4, n)


def test_falcon_training_step_matches_inner_fn_restatement():
    """FalconMamba trains through ``falcon_mamba_inner_fn`` (mamba_ssm's inner function with RMS
    weights for dt, B and C). transformers' sequential FalconMamba mixer normalises dt before
    ``dt_proj`` while that function normalises delta after it, so the training step is compared
    with the same model whose ``falcon_mamba_inner_fn`` is ``inner_fn_ref`` (plain PyTorch)."""
    from transformers.models.falcon_mamba import modeling_falcon_mamba as fm

    model = _build("falcon_mamba").train()
    ids = torch.randint(0, 80, (2, 50), generator=torch.Generator().manual_seed(2)).cuda()
    with _fast(model, "falcon_mamba"):
        assert fm.falcon_mamba_inner_fn is hf.mamba_inner_fn
        fast = _grads(model, ids)
        fm.falcon_mamba_inner_fn = inner_fn_ref
        ref = _grads(model, ids)
    _compare_grads(fast, ref)


def test_jamba_training_step_matches_sequential_path():
    """Jamba's mixer calls causal_conv1d_fn and selective_scan_fn itself (its inner RMS norms keep
    it off mamba_inner_fn); its training step is compared with the sequential mixer."""
    model = _build("jamba").train()
    ids = torch.randint(0, 80, (2, 50), generator=torch.Generator().manual_seed(2)).cuda()
    with _fast(model, "jamba"):
        fast = _grads(model, ids)
    with _slow(model, "jamba"):
        ref = _grads(model, ids)
    _compare_grads(fast, ref)


@pytest.mark.parametrize("family", FAMILIES)
def test_padded_batch_matches_sequential_path(family):
    """A left-padded batch (attention mask zeros at the start of one sequence)."""
    model = _build(family).eval()
    ids = torch.randint(0, 80, (2, 33), generator=torch.Generator().manual_seed(3)).cuda()
    mask = torch.ones_like(ids)
    mask[1, :9] = 0
    with torch.no_grad(), _fast(model, family):
        fast = model(ids, attention_mask=mask).logits
    with torch.no_grad(), _slow(model, family):
        ref = model(ids, attention_mask=mask).logits
    assert_close(fast, ref, 1e-4, 1e-4, "logits")


@pytest.mark.parametrize("family", ["falcon_mamba", "jamba"])
def test_cached_generation_matches_sequential_path(family):
    model = _build(family).eval()
    ids = torch.randint(0, 80, (2, 10), generator=torch.Generator().manual_seed(4)).cuda()
    kw = dict(max_new_tokens=6, do_sample=False)
    with torch.no_grad(), _fast(model, family):
        fast = model.generate(ids, **kw)
    with torch.no_grad(), _slow(model, family):
        ref = model.generate(ids, **kw)
    assert torch.equal(fast, ref)


def test_config3_prefill_matches_sequential_path():
    """BASELINE config 3 at full size: the random-init 130M MambaForCausalLM (24 layers, d_model
    768, d_inner 1536, dt_rank 48, vocab 50280, weights N(0, 0.02)), fp32 prefill of 1024 tokens,
    through the patched route against transformers' sequential mixer on the same GPU."""
    torch.manual_seed(0)
    cfg = transformers.MambaConfig(vocab_size=50280, hidden_size=768, state_size=16, num_hidden_layers=24, expand=2,
                                   conv_kernel=4, time_step_rank=48, use_mambapy=False, tie_word_embeddings=True,
                                   initializer_range=0.02)
    hf.patch_transformers()
    try:
        with torch.device("cuda"):
            model = transformers.MambaForCausalLM(cfg).float().eval()
    finally:
        hf.unpatch_transformers()
    ids = torch.randint(0, 50280, (1, 1024), generator=torch.Generator().manual_seed(1)).cuda()
    with torch.no_grad(), _fast(model, "mamba"):
        fast = model(ids).logits
    with torch.no_grad(), _slow(model, "mamba"):
        ref = model(ids).logits
    # fp32 through 24 layers: elementwise within 1e-3 relative, and the largest error small
    # against the largest logit
    assert_close(fast, ref, 1e-3, 1e-4, "logits", norm_tol=1e-4)
    del model
    torch.cuda.empty_cache()
