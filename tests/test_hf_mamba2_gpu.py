"""The Hugging Face route for Mamba-2 (an addition: the reference routes the Mamba-1 families only).

A small random-init ``Mamba2ForCausalLM`` (dstate 64, headdim 64) runs on CUDA through the patched
fast path -- prefill on ``mamba_chunk_scan_combined`` (the SSD kernel) and the conv1d kernel,
cached decoding on ``causal_conv1d_update`` and the wide-state ``selective_state_update`` -- and is
compared with the same model on transformers' own PyTorch mixer (``torch_forward``). The SSD kernel
multiplies in bf16, so the models are compared at bf16 tolerance (logits within 3e-2 of their
largest magnitude).
"""

import contextlib

import pytest
import torch

transformers = pytest.importorskip("transformers")

from mamba_cpu_b200 import hf  # noqa: E402

pytestmark = pytest.mark.gpu


def _build(dtype):
    torch.manual_seed(0)
    cfg = transformers.Mamba2Config(vocab_size=96, hidden_size=128, state_size=64, num_heads=4, head_dim=64,
                                    expand=2, n_groups=1, num_hidden_layers=2, conv_kernel=4, chunk_size=64)
    hf.patch_transformers()  # the mixers resolve their kernels when they are built
    try:
        model = transformers.Mamba2ForCausalLM(cfg)
    finally:
        hf.unpatch_transformers()
    return model.cuda().to(dtype).eval()


@contextlib.contextmanager
def _fast():
    hf.patch_transformers()
    try:
        yield
    finally:
        hf.unpatch_transformers()


def _close(got, want, tol, name):
    err = (got.float() - want.float()).abs().max().item()
    scale = want.float().abs().max().item()
    assert err <= tol * scale, f"{name}: max err {err:.3e} vs max |ref| {scale:.3e}"


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_mamba2_prefill_matches_sequential(dtype):
    model = _build(dtype)
    ids = torch.randint(0, 96, (2, 150), generator=torch.Generator().manual_seed(1)).cuda()
    with torch.no_grad():
        with _fast():
            fast = model(ids).logits
        slow = model(ids).logits  # unpatched: transformers' torch_forward
    torch.cuda.synchronize()
    _close(fast, slow, 3e-2, "logits")


def test_mamba2_cached_generation_matches_sequential():
    model = _build(torch.float32)
    ids = torch.randint(0, 96, (2, 70), generator=torch.Generator().manual_seed(2)).cuda()
    kw = dict(max_new_tokens=6, do_sample=False, output_scores=True, return_dict_in_generate=True)
    with torch.no_grad():
        with _fast():
            g_fast = model.generate(ids, **kw)
        g_slow = model.generate(ids, **kw)
    torch.cuda.synchronize()
    assert len(g_fast.scores) == len(g_slow.scores) == 6
    _close(g_fast.scores[0], g_slow.scores[0], 3e-2, "first generated step")
    if torch.equal(g_fast.sequences, g_slow.sequences):  # same prefixes: every decode step comparable
        for i, (a, b) in enumerate(zip(g_fast.scores, g_slow.scores)):
            _close(a, b, 3e-2, f"step {i}")


def test_mamba2_training_step_raises_clearly():
    """The SSD backward is not built: a training forward with gradients reaches it and raises."""
    model = _build(torch.bfloat16).train()
    ids = torch.randint(0, 96, (1, 64), generator=torch.Generator().manual_seed(3)).cuda()
    with _fast():
        out = model(ids, labels=ids)
        with pytest.raises(NotImplementedError):
            out.loss.backward()
