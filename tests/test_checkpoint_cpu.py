"""Checkpoints on the CPU: sharding a full Hugging Face state dict per rank, gathering it
back (gloo ranks), and the config.json + safetensors round trip, including a checkpoint
written by transformers itself."""
import json
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import free_port
from quantized_flash_communication_b200.models.config import LlamaConfig, get_config
from quantized_flash_communication_b200.models.llama import LlamaTP, TPContext


def _model(cfg, world, rank, init="full", seed=3):
    return LlamaTP(cfg, TPContext(device="cpu", world=world, rank=rank), "cpu", init=init, seed=seed)


@pytest.mark.parametrize("world", [2, 4])
def test_shards_of_a_full_state_dict_match_sharded_init(world):
    cfg = get_config("tiny")
    full = _model(cfg, 1, 0).state_dict()
    for r in range(world):
        ref = _model(cfg, world, r).state_dict()
        m = _model(cfg, world, r, init="empty")
        m.load_hf_state_dict(full)
        got = m.state_dict()
        assert set(got) == set(ref)
        for k in ref:
            assert torch.equal(got[k], ref[k]), (r, k)
        # the fused buffers the GEMMs read are updated through the views
        lay = m.model.layers[0]
        assert torch.equal(lay.self_attn.qkv_fused[: m.nq * m.hd], got["model.layers.0.self_attn.q_proj.weight"])
        assert torch.equal(lay.mlp.gate_up_fused[m.inter:], got["model.layers.0.mlp.up_proj.weight"])


def test_vocab_padding_of_the_lm_head():
    from dataclasses import replace
    cfg = replace(get_config("tiny"), vocab_size=1001)
    full = _model(cfg, 1, 0).state_dict()
    m1 = _model(cfg, 2, 1, init="empty")
    m1.load_hf_state_dict(full)
    head = m1.lm_head.weight
    assert head.shape[0] == 501
    assert torch.equal(head[:500], full["lm_head.weight"][501:])
    assert torch.count_nonzero(head[500]) == 0  # padded row never wins the argmax


def test_missing_weights_are_reported():
    cfg = get_config("tiny")
    full = _model(cfg, 1, 0).state_dict()
    del full["model.layers.1.mlp.down_proj.weight"]
    with pytest.raises(KeyError):
        _model(cfg, 2, 0, init="empty").load_hf_state_dict(full)


def test_save_and_load_round_trip(tmp_path):
    cfg = get_config("tiny")
    m = _model(cfg, 1, 0)
    m.save_pretrained(str(tmp_path))
    d = json.load(open(tmp_path / "config.json"))
    assert LlamaConfig.from_hf_dict(d, name=cfg.name) == cfg
    m2 = LlamaTP.from_pretrained(str(tmp_path), TPContext(device="cpu", world=2, rank=1), "cpu")
    ref = _model(cfg, 2, 1).state_dict()
    got = m2.state_dict()
    for k in ref:
        assert torch.equal(got[k], ref[k]), k


def test_loads_a_checkpoint_written_by_transformers(tmp_path):
    transformers = pytest.importorskip("transformers")
    hfc = transformers.LlamaConfig(hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                                   num_attention_heads=4, num_key_value_heads=2, vocab_size=300, head_dim=64,
                                   rms_norm_eps=1e-6, rope_theta=500000.0, max_position_embeddings=512,
                                   tie_word_embeddings=True)
    torch.manual_seed(0)
    hf = transformers.LlamaForCausalLM(hfc).to(torch.bfloat16)
    hf.save_pretrained(str(tmp_path), safe_serialization=True)
    sd = hf.state_dict()
    for world in (1, 2):
        for r in range(world):
            m = LlamaTP.from_pretrained(str(tmp_path), TPContext(device="cpu", world=world, rank=r), "cpu")
            assert m.cfg.tie_word_embeddings and m.cfg.head_dim == 64 and m.cfg.num_kv_heads == 2
            got = m.state_dict()
            q = got["model.layers.1.self_attn.q_proj.weight"]
            n = q.shape[0]
            assert torch.equal(q, sd["model.layers.1.self_attn.q_proj.weight"][r * n:(r + 1) * n])
            d = got["model.layers.0.mlp.down_proj.weight"]
            c = d.shape[1]
            assert torch.equal(d, sd["model.layers.0.mlp.down_proj.weight"][:, r * c:(r + 1) * c])
            v = m.v_local
            lm = got["lm_head.weight"]
            ref = sd["model.embed_tokens.weight"][r * v:(r + 1) * v]  # tied
            assert torch.equal(lm[: ref.shape[0]], ref)
            assert torch.equal(got["model.norm.weight"], sd["model.norm.weight"])


def _gather_worker(rank, world, port, path, results):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60))
    try:
        cfg = get_config("tiny")
        tp = TPContext(device="cpu", ar_backend="nccl")  # gloo group: plain torch.distributed collectives
        m = LlamaTP(cfg, tp, "cpu", init="full", seed=3)
        full = m.full_state_dict()
        ref = _model(cfg, 1, 0).state_dict()
        results[rank] = all(torch.equal(full[k], ref[k]) for k in ref) and set(full) == set(ref)
        m.save_pretrained(path)
    finally:
        dist.destroy_process_group()


def test_full_state_dict_gathers_the_shards(tmp_path):
    world = 2
    results = mp.Manager().dict()
    mp.spawn(_gather_worker, args=(world, free_port(), str(tmp_path), results), nprocs=world, join=True)
    assert all(results[r] for r in range(world))
    m = LlamaTP.from_pretrained(str(tmp_path), TPContext(device="cpu", world=1), "cpu")
    ref = _model(get_config("tiny"), 1, 0).state_dict()
    got = m.state_dict()
    assert all(torch.equal(got[k], ref[k]) for k in ref)
