"""The SDPA patch inside a real HuggingFace Llama model (randomly initialised
tiny configuration: no weights are needed), as the reference's
llama_attention_replacement example runs it with a downloaded model.

A left-padded batch exercises the padded-mask route, a prompt without padding
the plain causal route, and one KV-cache decode step the Nq != Nk route; the
logits must match the unpatched model's on every real (non-padding) token
within fp16 tolerance.  A training step checks the autograd route (loss and
attention-weight gradients against the unpatched model).
"""
import pytest
import torch

from flash_attention_sm75 import llama_attention_replacement as patch

pytestmark = pytest.mark.gpu


def _tiny_llama(seed=0):
    from transformers import LlamaConfig, LlamaForCausalLM
    cfg = LlamaConfig(vocab_size=512, hidden_size=256, intermediate_size=512,
                      num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                      head_dim=64, max_position_embeddings=1024)
    torch.manual_seed(seed)
    model = LlamaForCausalLM(cfg).to(device="cuda", dtype=torch.float16)
    model.config._attn_implementation = "sdpa"
    return model.eval()


def _logits(model, ids, mask):
    with torch.no_grad():
        return model(input_ids=ids, attention_mask=mask).logits.float()


def test_llama_forward_with_padding(sm100):
    model = _tiny_llama()
    g = torch.Generator().manual_seed(1)
    B, N = 3, 200
    ids = torch.randint(0, 512, (B, N), generator=g).cuda()
    mask = torch.ones(B, N, dtype=torch.long, device="cuda")
    mask[1, :37] = 0    # left padding
    mask[2, :150] = 0
    ref = _logits(model, ids, mask)
    patch.reset_stats()
    patch.apply_patch()
    try:
        out = _logits(model, ids, mask)
        plain = _logits(model, ids[:1], mask[:1])  # no padding
    finally:
        patch.remove_patch()
    s = patch.patch_stats()
    real = mask.bool()
    err = (out - ref).abs()[real]
    assert err.max().item() < 5e-2, err.max().item()
    assert (plain - ref[:1]).abs().max().item() < 5e-2
    assert s["flash"] == s["total"] and s["fallback"] == 0, s
    assert s["flash_masked"] >= 2, s  # both layers of the padded batch


def test_llama_decode_step(sm100):
    """Prefill, then one cached decode step: the patch serves the step's
    Nq = 1 call through the KV-cache kernel."""
    model = _tiny_llama(seed=2)
    g = torch.Generator().manual_seed(3)
    ids = torch.randint(0, 512, (2, 96), generator=g).cuda()
    nxt = torch.randint(0, 512, (2, 1), generator=g).cuda()

    def run():
        with torch.no_grad():
            o = model(input_ids=ids, use_cache=True)
            step = model(input_ids=nxt, past_key_values=o.past_key_values, use_cache=True)
        return o.logits.float(), step.logits.float()

    ref_pre, ref_dec = run()
    patch.reset_stats()
    patch.apply_patch()
    try:
        pre, dec = run()
    finally:
        patch.remove_patch()
    s = patch.patch_stats()
    assert (pre - ref_pre).abs().max().item() < 5e-2
    assert (dec - ref_dec).abs().max().item() < 5e-2
    assert s["flash_kvcache"] >= 2 and s["fallback"] == 0, s


def test_llama_training_step(sm100):
    """A training step through the patch: the causal GQA attention calls run the
    forward and backward kernels (the reference's patch raised in backward);
    loss and gradients match the unpatched model's."""
    model = _tiny_llama(seed=4)
    g = torch.Generator().manual_seed(5)
    ids = torch.randint(0, 512, (2, 160), generator=g).cuda()

    def step():
        model.zero_grad(set_to_none=True)
        loss = model(input_ids=ids, labels=ids).loss
        loss.backward()
        return loss.item(), {n: p.grad.float().clone() for n, p in model.named_parameters()
                             if p.grad is not None and "self_attn" in n}

    ref_loss, ref_g = step()
    patch.reset_stats()
    patch.apply_patch()
    try:
        loss, grads = step()
    finally:
        patch.remove_patch()
    s = patch.patch_stats()
    assert s["flash_autograd"] == 2 and s["fallback"] == 0, s
    assert abs(loss - ref_loss) < 1e-2 * abs(ref_loss)
    for n, gr in ref_g.items():
        err = (grads[n] - gr).abs().max().item()
        assert err <= 3e-2 * gr.abs().max().item() + 1e-5, (n, err, gr.abs().max().item())


def test_llama_training_step_padded(sm100):
    """A training step on a left-padded batch: the masked attention calls run
    the padded forward and backward kernels."""
    model = _tiny_llama(seed=6)
    g = torch.Generator().manual_seed(7)
    ids = torch.randint(0, 512, (3, 144), generator=g).cuda()
    mask = torch.ones(3, 144, dtype=torch.long, device="cuda")
    mask[1, :40] = 0
    mask[2, :100] = 0
    # labels shift by one: the first real token is predicted from the last
    # padding position, whose output SDPA leaves implementation-defined, so it
    # is excluded too; every remaining loss term depends on real rows only
    labels = ids.masked_fill(mask == 0, -100)
    labels[1, 40] = -100
    labels[2, 100] = -100

    def step():
        model.zero_grad(set_to_none=True)
        loss = model(input_ids=ids, attention_mask=mask, labels=labels).loss
        loss.backward()
        return loss.item(), {n: p.grad.float().clone() for n, p in model.named_parameters()
                             if p.grad is not None and "self_attn" in n}

    ref_loss, ref_g = step()
    patch.reset_stats()
    patch.apply_patch()
    try:
        loss, grads = step()
    finally:
        patch.remove_patch()
    s = patch.patch_stats()
    assert s["flash_autograd"] == 2 and s["flash_masked"] == 2 and s["fallback"] == 0, s
    assert abs(loss - ref_loss) < 1e-2 * abs(ref_loss)
    for n, gr in ref_g.items():
        err = (grads[n] - gr).abs().max().item()
        assert err <= 3e-2 * gr.abs().max().item() + 1e-5, (n, err, gr.abs().max().item())
