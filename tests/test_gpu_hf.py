"""transformers integration on a B200: a small random-weight Llama (head_dim
128, GQA 2) run with attn_implementation set to the ATFlash attention function
gives the same prefill and decode logits as SDPA when the window is off, and
the window at k=inf is bit-identical to no window (the reference's harness
contract, e2e_pipeline/atflash_e2e_fafi.py:81-120)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _models():
    from transformers import LlamaConfig, LlamaForCausalLM
    import atflash.hf
    cfg = LlamaConfig(vocab_size=256, hidden_size=512, intermediate_size=1024, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, head_dim=128,
                      max_position_embeddings=4096, rope_theta=10000.0)
    torch.manual_seed(0)
    ref = LlamaForCausalLM(cfg).to(torch.bfloat16).cuda().eval()
    ref.set_attn_implementation("sdpa")
    atf = LlamaForCausalLM(cfg).to(torch.bfloat16).cuda().eval()
    atf.load_state_dict(ref.state_dict())
    name = atflash.hf.register()
    atf.set_attn_implementation(name)
    return ref, atf


def _rel(a, b):
    return ((a.float() - b.float()).abs().max() / b.float().abs().max()).item()


@torch.inference_mode()
def test_dense_prefill_and_decode_match_sdpa():
    ref, atf = _models()
    ids = torch.randint(0, 256, (2, 300), generator=torch.Generator().manual_seed(1)).cuda()
    r = ref(input_ids=ids, use_cache=True)
    a = atf(input_ids=ids, use_cache=True)
    assert _rel(a.logits, r.logits) < 3e-2
    nxt = torch.randint(0, 256, (2, 1), generator=torch.Generator().manual_seed(2)).cuda()
    r2 = ref(input_ids=nxt, past_key_values=r.past_key_values, use_cache=True)
    a2 = atf(input_ids=nxt, past_key_values=a.past_key_values, use_cache=True)
    assert _rel(a2.logits, r2.logits) < 3e-2
    import atflash
    assert atflash.check_device_errors() == 0


@torch.inference_mode()
def test_window_kinf_is_bitwise_dense_and_k2_runs():
    import atflash
    import atflash.hf
    ref, atf = _models()
    ids = torch.randint(0, 256, (1, 260), generator=torch.Generator().manual_seed(3)).cuda()
    atflash.hf.configure(None, None)
    dense = atf(input_ids=ids, use_cache=True)
    pk, dk = atflash.hf.window_tables_for_model(atf, float("inf"), float("inf"))
    atflash.hf.configure(pk, dk)
    kinf = atf(input_ids=ids, use_cache=True)
    assert torch.equal(dense.logits, kinf.logits)
    pk, dk = atflash.hf.window_tables_for_model(atf, 2.0, 2.0)
    atflash.hf.configure(pk, dk)
    win = atf(input_ids=ids, use_cache=True)
    step = atf(input_ids=ids[:, -1:], past_key_values=win.past_key_values, use_cache=True)
    assert torch.isfinite(win.logits).all() and torch.isfinite(step.logits).all()
    assert atflash.check_device_errors() == 0
    atflash.hf.configure(None, None)
