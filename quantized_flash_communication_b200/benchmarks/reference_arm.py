"""Harness for the reference's own code path (the unmodified files in ``baseline/_ref``).

Builds a Hugging Face ``LlamaForCausalLM`` of a benchmark architecture with random
N(0, 0.02) weights in fp16 (the reference's dtype), then applies the reference's
``inject_ultimate_layers`` (MLP-only tensor parallelism, reference main.py:25-39) and
switches every injected MLP to its ``flash_all_reduce`` (communication.py:7-97) with the
given bits / group size / mode, as the reference's tables and QA test do (main.py:93-97,
inference.py:9-12).  Nothing of this package's models, kernels or engine is on that path:
only the architecture's numbers come from ``models.config``.
"""
from __future__ import annotations

import os
import sys
import types

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
REF_DIR = os.path.join(ROOT, "baseline", "_ref")

__all__ = ["REF_DIR", "reference_available", "import_reference", "build_reference_model"]


def reference_available() -> bool:
    return os.path.isfile(os.path.join(REF_DIR, "communication.py"))


def import_reference():
    """The reference's ``main`` module.  Its ``utils`` import names a module the reference
    does not ship (main.py:17); a stand-in with the three imported names is provided."""
    import torch
    if "utils" not in sys.modules or not hasattr(sys.modules["utils"], "set_seed"):
        stub = types.ModuleType("utils")
        stub.setup_ddp = lambda *a, **k: None
        stub.cleanup_ddp = lambda *a, **k: None
        stub.set_seed = lambda s=42: torch.manual_seed(s)
        sys.modules["utils"] = stub
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    import main as ref_main  # noqa: E402  (reference, unmodified)
    return ref_main


def build_reference_model(cfg, dev, rank: int, world: int, bits: int = 8, group_size: int = 128,
                          quant_type: str = "asym", seed: int = 1234):
    import torch
    from transformers import LlamaConfig as HFConfig, LlamaForCausalLM
    ref_main = import_reference()
    hf = HFConfig(hidden_size=cfg.hidden_size, intermediate_size=cfg.intermediate_size,
                  num_hidden_layers=cfg.num_layers, num_attention_heads=cfg.num_heads,
                  num_key_value_heads=cfg.num_kv_heads, vocab_size=cfg.vocab_size, rms_norm_eps=cfg.rms_eps,
                  rope_theta=cfg.rope_theta, max_position_embeddings=cfg.max_position, initializer_range=0.02,
                  tie_word_embeddings=False)
    torch.manual_seed(seed)
    prev = torch.get_default_dtype()
    torch.set_default_dtype(torch.float16)
    with torch.device(dev):
        model = LlamaForCausalLM(hf)
    torch.set_default_dtype(prev)
    model.eval()
    ref_main.inject_ultimate_layers(model, rank, world)
    for layer in model.model.layers:
        layer.mlp.mode = "flash"
        layer.mlp.bits = bits
        layer.mlp.group_size = group_size
        layer.mlp.quant_type = quant_type
    return model
