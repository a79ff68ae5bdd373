"""Tensor-parallel Llama (TP=1) vs Hugging Face LlamaForCausalLM with the same weights."""
import pytest
import torch

from quantized_flash_communication_b200.models.config import get_config
from quantized_flash_communication_b200.models.llama import LlamaTP, TPContext
from quantized_flash_communication_b200.quantization import rel_l2

pytestmark = pytest.mark.gpu


def _hf(cfg, sd, dev):
    from transformers import LlamaConfig as HFC, LlamaForCausalLM
    hfc = HFC(hidden_size=cfg.hidden_size, intermediate_size=cfg.intermediate_size, num_hidden_layers=cfg.num_layers,
              num_attention_heads=cfg.num_heads, num_key_value_heads=cfg.num_kv_heads, vocab_size=cfg.vocab_size,
              head_dim=cfg.head_dim, rms_norm_eps=cfg.rms_eps, rope_theta=cfg.rope_theta,
              max_position_embeddings=cfg.max_position, tie_word_embeddings=False)
    with torch.device(dev):
        hf = LlamaForCausalLM(hfc)
    # Cast parameters only: the rotary inverse-frequency buffers stay fp32, as after
    # from_pretrained (a blanket .to(bfloat16) would round the rotation angles too).
    dtype = next(iter(sd.values())).dtype
    for p in hf.parameters():
        p.data = p.data.to(dtype)
    missing, unexpected = hf.load_state_dict(sd, strict=False)
    assert not unexpected and all("rotary" in k for k in missing)
    return hf.eval()


@pytest.mark.parametrize("name", ["tiny", "tiny-mha"])
def test_prefill_and_decode_match_hf(cuda_device, name):
    """Our bf16 model must be as close to an fp32 oracle as Hugging Face's bf16 model is."""
    cfg = get_config(name)
    m = LlamaTP(cfg, TPContext(device=cuda_device), cuda_device, init="full", seed=11, init_std=0.05)
    sd = m.state_dict()
    hf = _hf(cfg, sd, cuda_device)
    hf32 = _hf(cfg, {k: v.float() for k, v in sd.items()}, cuda_device).float()
    B, S = 3, 100
    ids = torch.randint(0, cfg.vocab_size, (B, S), device=cuda_device)
    cache = m.new_cache(B, S + 4)
    tok, x_last = m.prefill(ids, cache, return_last_hidden=True)
    with torch.no_grad():
        out = hf(ids, output_hidden_states=True)
        out32 = hf32(ids, output_hidden_states=True)
    ref32 = out32.hidden_states[-1][:, -1].float()
    err_ours = rel_l2(x_last.float(), ref32)
    err_hf = rel_l2(out.hidden_states[-1][:, -1].float(), ref32)
    assert err_ours <= 1.5 * err_hf + 0.01, (err_ours, err_hf)
    ref_logits = out32.logits[:, -1].float()
    ours_logits = (x_last.float() @ m.lm_head.weight.float().T)
    assert rel_l2(ours_logits, ref_logits) <= 1.5 * rel_l2(out.logits[:, -1].float(), ref_logits) + 0.01
    # greedy tokens agree with the fp32 oracle where its top-2 margin is clear
    top2 = ref_logits.topk(2, -1).values
    clear = (top2[:, 0] - top2[:, 1]) > 0.05 * top2[:, 0].abs().clamp_min(1)
    assert torch.equal(tok[clear], ref_logits.argmax(-1)[clear])
    # one decode step == the oracle on the extended sequence
    tok2 = m.decode_step(tok, cache)
    with torch.no_grad():
        ref2 = hf32(torch.cat([ids, tok.view(B, 1)], 1)).logits[:, -1].float()
    top2 = ref2.topk(2, -1).values
    clear = (top2[:, 0] - top2[:, 1]) > 0.05 * top2[:, 0].abs().clamp_min(1)
    assert torch.equal(tok2[clear], ref2.argmax(-1)[clear])
    assert int(cache.seq_lens[0]) == S + 1


@pytest.mark.parametrize("nq,nkv,hd,page,dtype", [
    (16, 4, 128, 64, torch.bfloat16),
    (8, 8, 128, 16, torch.bfloat16),
    (8, 4, 128, 16, torch.float16),
    (32, 4, 128, 32, torch.bfloat16),
    (16, 16, 64, 16, torch.float16),
    (8, 4, 64, 64, torch.bfloat16),
    (16, 4, 64, 16, torch.bfloat16),
    (16, 2, 64, 16, torch.float16),
])
def test_decode_attention_vs_torch(cuda_device, nq, nkv, hd, page, dtype):
    from quantized_flash_communication_b200.ops.attention import decode_attention
    B = 5
    lens = torch.tensor([1, 63, 64, 700, 1500], dtype=torch.int32, device=cuda_device)
    pps = (1500 + page - 1) // page + 1
    kc = torch.randn(B * pps, nkv, page, hd, device=cuda_device, dtype=dtype)
    vc = torch.randn_like(kc)
    bt = torch.randperm(B * pps, device=cuda_device, dtype=torch.int32).view(B, pps).contiguous()
    q = torch.randn(B, nq * hd, device=cuda_device, dtype=dtype) * 2
    o = decode_attention(q, kc, vc, bt, lens, nq, nkv, hd)
    for b in range(B):
        L = int(lens[b])
        pages = bt[b, : (L + page - 1) // page].long()
        K = kc[pages].permute(1, 0, 2, 3).reshape(nkv, -1, hd)[:, :L].float()
        V = vc[pages].permute(1, 0, 2, 3).reshape(nkv, -1, hd)[:, :L].float()
        qq = q[b].view(nq, hd).float()
        K = K.repeat_interleave(nq // nkv, 0)
        V = V.repeat_interleave(nq // nkv, 0)
        p = torch.softmax((qq.unsqueeze(1) @ K.transpose(1, 2)) / hd ** 0.5, -1)
        ref = (p @ V).squeeze(1).reshape(-1)
        assert rel_l2(o[b].float(), ref) < 0.01, b


def test_ultimate_tp_mlp_single_rank(cuda_device):
    from quantized_flash_communication_b200.model import Ultimate_TP_MLP
    cfg = get_config("tiny")
    mlp = Ultimate_TP_MLP(cfg, 1).to(cuda_device, torch.bfloat16)
    x = torch.randn(2, 7, cfg.hidden_size, device=cuda_device, dtype=torch.bfloat16)
    y = mlp(x)
    ref = mlp.down_proj(torch.nn.functional.silu(mlp.gate_proj(x)) * mlp.up_proj(x))
    assert rel_l2(y.float(), ref.float()) < 0.02


def test_loss_matches_hf_cross_entropy(cuda_device):
    cfg = get_config("tiny")
    m = LlamaTP(cfg, TPContext(device=cuda_device), cuda_device, init="full", seed=2)
    hf32 = _hf(cfg, {k: v.float() for k, v in m.state_dict().items()}, cuda_device).float()
    ids = torch.randint(0, cfg.vocab_size, (2, 50), device=cuda_device)
    ours = float(m.loss(ids))
    with torch.no_grad():
        logits = hf32(ids).logits[:, :-1].reshape(-1, cfg.vocab_size)
    ref = float(torch.nn.functional.cross_entropy(logits, ids[:, 1:].reshape(-1)))
    assert abs(ours - ref) / ref < 0.02, (ours, ref)


def test_reference_tables_and_qa_entry_points(cuda_device):
    from quantized_flash_communication_b200.inference import run_qa_test
    from quantized_flash_communication_b200.main import benchmark_all_tables
    cfg = get_config("tiny")
    m = LlamaTP(cfg, TPContext(device=cuda_device), cuda_device, init="shard", seed=1)
    res = benchmark_all_tables(m, None, cuda_device, 0, block_list=(512, 128), volumes_mb=(1,), batches=(2,), seq=16)
    assert len(res["table1"]) == cfg.num_layers and len(res["table2"]) == 2 and len(res["table4"]) == 1
    assert all(r[1] > 0 for r in res["table1"])
    toks, ms = run_qa_test(m, None, cuda_device, 0, max_new_tokens=4, verbose=False)
    assert toks.shape == (1, 4) and ms > 0


def test_cuda_graph_prefill_and_decode_match_eager(cuda_device):
    cfg = get_config("tiny")
    m = LlamaTP(cfg, TPContext(device=cuda_device), cuda_device, init="full", seed=4)
    B, S = 2, 96
    ids = torch.randint(0, cfg.vocab_size, (B, S), device=cuda_device)
    c1 = m.new_cache(B, S + 3)
    t_eager = m.prefill(ids, c1)
    d_eager = m.decode_step(t_eager, c1)
    c2 = m.new_cache(B, S + 3)
    g = m.capture_prefill(B, S, c2)
    t_graph = g(ids).clone()
    assert torch.equal(t_graph, t_eager)
    dg = m.capture_decode(c2)
    assert int(c2.seq_lens[0]) == S
    d_graph = dg(t_graph).clone()
    assert torch.equal(d_graph, d_eager) and int(c2.seq_lens[0]) == S + 1
    g.release()
    dg.release()
