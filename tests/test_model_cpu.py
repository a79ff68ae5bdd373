"""Model construction on CPU: Hugging Face state-dict layout and tensor-parallel shards."""
import torch

from quantized_flash_communication_b200.models.config import get_config
from quantized_flash_communication_b200.models.llama import LlamaTP, TPContext


def test_state_dict_layout_tp1():
    cfg = get_config("tiny")
    m = LlamaTP(cfg, TPContext(device="cpu"), device="cpu", init="full", seed=3)
    sd = m.state_dict()
    H, hd = cfg.hidden_size, cfg.head_dim
    assert sd["model.embed_tokens.weight"].shape == (cfg.vocab_size, H)
    assert sd["model.layers.0.self_attn.q_proj.weight"].shape == (cfg.num_heads * hd, H)
    assert sd["model.layers.0.self_attn.k_proj.weight"].shape == (cfg.num_kv_heads * hd, H)
    assert sd["model.layers.0.self_attn.o_proj.weight"].shape == (H, cfg.num_heads * hd)
    assert sd["model.layers.1.mlp.gate_proj.weight"].shape == (cfg.intermediate_size, H)
    assert sd["model.layers.1.mlp.down_proj.weight"].shape == (H, cfg.intermediate_size)
    assert sd["model.norm.weight"].shape == (H,)
    assert sd["lm_head.weight"].shape == (cfg.vocab_size, H)
    assert not any("fused" in k for k in sd)
    # HF's module tree has exactly these parameter names
    from transformers import LlamaConfig as HFC, LlamaForCausalLM
    hf = LlamaForCausalLM(HFC(hidden_size=H, intermediate_size=cfg.intermediate_size, num_hidden_layers=cfg.num_layers,
                              num_attention_heads=cfg.num_heads, num_key_value_heads=cfg.num_kv_heads,
                              vocab_size=cfg.vocab_size, head_dim=hd, tie_word_embeddings=False))
    assert set(hf.state_dict().keys()) - {k for k in hf.state_dict() if "rotary" in k} == set(sd.keys())


def test_fused_views_share_storage():
    m = LlamaTP(get_config("tiny"), TPContext(device="cpu"), device="cpu")
    lay = m.model.layers[0]
    lay.self_attn.k_proj.weight.data.fill_(7.0)
    nq = m.nq * m.hd
    assert bool((lay.self_attn.qkv_fused[nq:nq + m.nkv * m.hd] == 7.0).all())
    m.load_state_dict({k: torch.zeros_like(v) for k, v in m.state_dict().items()})
    assert float(lay.mlp.gate_up_fused.abs().sum()) == 0.0


def test_tp_shards_tile_the_full_weights():
    cfg = get_config("tiny")
    full = LlamaTP(cfg, TPContext(device="cpu"), device="cpu", init="full", seed=5).state_dict()
    W = 2
    shards = [LlamaTP(cfg, TPContext(device="cpu", world=W, rank=r), device="cpu", init="full", seed=5).state_dict()
              for r in range(W)]
    for name in ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "mlp.gate_proj", "mlp.up_proj"):
        k = f"model.layers.1.{name}.weight"
        assert torch.equal(torch.cat([s[k] for s in shards], 0), full[k])
    for name in ("self_attn.o_proj", "mlp.down_proj"):
        k = f"model.layers.0.{name}.weight"
        assert torch.equal(torch.cat([s[k] for s in shards], 1), full[k])
    assert torch.equal(torch.cat([s["lm_head.weight"] for s in shards], 0)[:cfg.vocab_size], full["lm_head.weight"])
    assert torch.equal(shards[1]["model.embed_tokens.weight"], full["model.embed_tokens.weight"])


def test_configs_match_the_benchmark_configurations():
    """The architectures the benchmarks run are the ones the benchmark configurations name:
    Llama-2-7B (32 layers, hidden 4096, 32 heads, FFN 11008, vocab 32000), Llama-3-8B
    (32 / 4096 / 32 q + 8 kv heads / 14336 / 128256) and Llama-3-70B (80 / 8192 / 64 + 8 /
    28672 / 128256); head_dim 128 everywhere, and every head count divides by 8 ranks."""
    from quantized_flash_communication_b200.models.config import get_config
    want = {"llama2-7b": (32, 4096, 32, 32, 11008, 32000), "llama3-8b": (32, 4096, 32, 8, 14336, 128256),
            "llama3-70b": (80, 8192, 64, 8, 28672, 128256)}
    for name, (L, H, nq, nkv, inter, vocab) in want.items():
        c = get_config(name)
        assert (c.num_layers, c.hidden_size, c.num_heads, c.num_kv_heads, c.intermediate_size,
                c.vocab_size) == (L, H, nq, nkv, inter, vocab), name
        assert c.head_dim == 128 and nq % 8 == 0 and nkv % 8 == 0 and inter % 8 == 0, name
