"""Tensor-parallel Llama (Llama-2 / Llama-3 architectures) on the sm_100a kernels.

The reference tensor-parallelises only the MLP of a Hugging Face model and replicates
attention on every rank (model.py:8-57, main.py:25-39).  This model shards the whole
decoder layer Megatron-style, one process per GPU:

* q/k/v projections column-parallel by head, o_proj row-parallel;
* gate/up column-parallel, down_proj row-parallel;
* embedding replicated, lm_head vocab-parallel (argmax combined across ranks);
* one all-reduce after o_proj and one after down_proj, through the fused quantized
  kernel (``parallel/quant_allreduce.py``), NCCL (baseline) or nothing at TP=1.

Parameters carry Hugging Face's state-dict names (``model.layers.{i}.self_attn.q_proj
.weight`` ...) holding this rank's shard; q/k/v and gate/up are views into one fused
buffer per layer, which the fused GEMMs read.  Every op on the forward path is a kernel
of this package: tcgen05 GEMMs (with SwiGLU / residual epilogues), RMSNorm with fused
residual add, RoPE + paged KV-cache write, attention, embedding and argmax.
"""
from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Optional

import torch
import torch.distributed as dist
import torch.nn as nn

from ..ops import attention as A
from ..ops import gemm as G
from ..ops import layers as L
from ..parallel.quant_allreduce import QuantAllReduce
from ..utils.trace import maybe_region
from .config import LlamaConfig, get_config
from .sampling import Sampler

__all__ = ["TPContext", "LlamaTP", "KVCache", "Sampler", "smoke_forward"]


# ------------------------------------------------------------------------------------------
# Tensor-parallel context
# ------------------------------------------------------------------------------------------
class TPContext:
    """Process group of a tensor-parallel model and the all-reduce it uses.

    ``ar_backend``: "qfc" (fused quantized kernel over peer memory), "nccl" (bf16 NCCL
    all-reduce, the baseline) or "staged" (the reference's collective structure).
    ``bits``: 16 / 8 / 6 / 4 as in the reference's flash_all_reduce.
    """

    def __init__(self, group: Optional[dist.ProcessGroup] = None, device=None, ar_backend: str = "qfc",
                 bits: int = 8, group_size: int = 128, quant_type: str = "asym", algo: str = "auto",
                 reserve_tokens: int = 0, hidden_size: int = 0, world: Optional[int] = None,
                 rank: Optional[int] = None, fuse_gemm: bool = True, seq_parallel: Optional[bool] = None):
        self.group = group
        if world is not None:  # explicit (e.g. building one shard offline); no communication
            self.world, self.rank = world, rank or 0
            ar_backend = "none" if world > 1 else ar_backend
        elif dist.is_available() and dist.is_initialized():
            self.world = dist.get_world_size(group)
            self.rank = dist.get_rank(group)
        else:
            self.world, self.rank = 1, 0
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.ar_backend = ar_backend
        self.bits = bits
        self.group_size = group_size
        self.quant_type = quant_type
        self.algo = algo
        # quantize-and-scatter inside the row-parallel GEMMs' epilogue (two-shot, group 128)
        self.fuse_gemm = fuse_gemm and group_size == 128
        self.fuse_min_rows = 256  # below this, messages go one-shot through the plain kernel
        # The fused epilogue stores every tile's quantized rows into their owners' slots, so
        # at 8 ranks 7/8 of every tile leaves over NVLink from the GEMM's epilogue, whose
        # store stream then paces the GEMM, and the GEMM followed by the standalone
        # all-reduce kernel is faster.  Measured on
        # the Llama-2-7B prefill step (8 x 1024 tokens, INT8, sequence-parallel residual):
        # 4 ranks 30.25 ms fused vs 32.18 ms unfused, 8 ranks 24.56 ms vs 23.20 ms.
        self.fuse_max_world = int(os.environ.get("QFC_FUSE_MAX_WORLD", "4"))
        self.timer = None  # utils.trace.OpTimer shared with the model when attached
        self.ar: Optional[QuantAllReduce] = None
        if self.world > 1 and ar_backend == "qfc":
            self.ar = QuantAllReduce(group, self.device, bits=bits, group_size=group_size, quant_type=quant_type,
                                     algo=algo)
            if reserve_tokens and hidden_size:
                self.ar.reserve(reserve_tokens * hidden_size, torch.bfloat16, bits_options=(bits, 16))
        # Sequence-parallel residual stream for prefill: each rank keeps rows
        # [r*R, (r+1)*R) of the residual and the row-parallel all-reduces also add the
        # residual and apply the next RMSNorm on those rows (csrc/allreduce_norm.cuh), so
        # only the normalised activations are all-gathered.  Default (seq_parallel=None):
        # on from ``sp_min_world`` ranks (QFC_SEQ_PARALLEL=1 / 0 forces it on / off).  On the
        # Llama-2-7B prefill step (8 x 1024 tokens, INT8) it takes the fused-epilogue step
        # from 53.12 to 51.17 ms at 2 ranks and from 32.59 to 30.25 ms at 4, and the
        # unfused step from 24.66 to 23.20 ms at 8.
        self.sp_min_world = int(os.environ.get("QFC_SP_MIN_WORLD", "2"))
        if seq_parallel is None:
            env = os.environ.get("QFC_SEQ_PARALLEL")
            seq_parallel = (env == "1") if env is not None else self.world >= self.sp_min_world
        self.seq_parallel = bool(seq_parallel) and self.ar is not None and group_size == 128
        if self.seq_parallel and reserve_tokens and hidden_size:
            self.ar.reserve_rows(reserve_tokens, hidden_size, bits_options=(bits, 16))

    def sp_active(self, rows: int, hidden: int) -> bool:
        """Whether a step of ``rows`` tokens runs with the sequence-parallel residual."""
        return (self.seq_parallel and self.ar is not None and self.ar_backend == "qfc" and self.group_size == 128
                and rows >= self.fuse_min_rows and hidden % 256 == 0)

    def sp_rows(self, rows: int):
        """(rows per rank R, first row, rows owned) of this rank's residual shard."""
        R = (rows + self.world - 1) // self.world
        lo = self.rank * R
        return R, lo, max(0, min(rows, lo + R) - lo)

    def linear_all_reduce_norm(self, x: torch.Tensor, w: torch.Tensor, h_shard: torch.Tensor,
                               norm_w: torch.Tensor, eps: float) -> torch.Tensor:
        """Sequence-parallel ``h_shard += all_reduce(x @ w.T)`` (own rows) and the full
        ``rmsnorm(h) * norm_w`` of every row, gathered from the row owners."""
        if (self.world <= self.fuse_max_world and self.fuse_gemm and w.shape[0] % 128 == 0):
            return self.ar.gemm_all_reduce_norm(x, w, h_shard, norm_w, eps, bits=self.bits,
                                                quant_type=self.quant_type)
        with maybe_region(self.timer, "  (gemm part)"):
            p = G.linear(x, w)
        with maybe_region(self.timer, "  (allreduce+norm part)"):
            return self.ar.all_reduce_norm(p, h_shard, norm_w, eps, bits=self.bits, quant_type=self.quant_type)

    def configure(self, bits: Optional[int] = None, group_size: Optional[int] = None,
                  quant_type: Optional[str] = None, backend: Optional[str] = None):
        """Change the all-reduce settings at run time (the reference mutates ``mode``, ``bits``,
        ``group_size`` and ``quant_type`` of every layer, main.py:93-97, 166-170)."""
        if bits is not None:
            self.bits = bits
        if group_size is not None:
            self.group_size = group_size
        if quant_type is not None:
            self.quant_type = quant_type
        if backend is not None:
            if backend == "qfc" and self.ar is None and self.world > 1:
                self.ar = QuantAllReduce(self.group, self.device, bits=self.bits, group_size=128,
                                         quant_type=self.quant_type, algo=self.algo)
            self.ar_backend = backend

    def all_reduce(self, x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        if self.world == 1:
            return x
        if self.ar_backend == "qfc" and 8 <= self.group_size <= 256:
            return self.ar(x, out=out, bits=self.bits, group_size=self.group_size, quant_type=self.quant_type)
        if self.ar_backend == "qfc":  # groups above 256: the staged (torch.distributed) path
            from ..parallel.staged import staged_all_reduce
            return staged_all_reduce(x, self.bits, self.group_size, self.quant_type, torch.float16, self.group, x.dtype)
        if self.ar_backend == "nccl":
            dist.all_reduce(x, group=self.group)
            return x
        if self.ar_backend == "staged":
            from ..parallel.staged import staged_all_reduce
            return staged_all_reduce(x, self.bits, self.group_size, self.quant_type, torch.float16, self.group, x.dtype)
        raise ValueError(f"unknown ar_backend {self.ar_backend!r}")

    def linear_all_reduce(self, x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        """``all_reduce(x @ w.T)`` for a row-parallel layer (o_proj, down_proj)."""
        if (self.world > 1 and self.world <= self.fuse_max_world and self.ar_backend == "qfc" and self.fuse_gemm
                and self.group_size == 128 and x.shape[0] >= self.fuse_min_rows and w.shape[0] % 128 == 0):
            return self.ar.gemm_all_reduce(x, w, bits=self.bits, quant_type=self.quant_type)
        with maybe_region(self.timer, "  (gemm part)"):
            p = G.linear(x, w)
        with maybe_region(self.timer, "  (allreduce part)"):
            return self.all_reduce(p, out=p)

    def gather_vocab(self, logits: torch.Tensor) -> torch.Tensor:
        """Full-vocabulary logits [B, W * V_local] from every rank's vocabulary slice."""
        if self.world == 1:
            return logits
        B, V = logits.shape
        buf = torch.empty(self.world, B, V, dtype=logits.dtype, device=logits.device)
        dist.all_gather_into_tensor(buf, logits.contiguous(), group=self.group)
        return buf.permute(1, 0, 2).reshape(B, self.world * V)

    def gather_argmax(self, val: torch.Tensor, idx: torch.Tensor) -> torch.Tensor:
        """Global argmax from per-rank (max value, index) pairs; ties go to the lower index."""
        if self.world == 1:
            return idx
        B = val.numel()
        if self.ar is not None and B <= 512:
            return self.ar.argmax(val, idx)  # one kernel over peer memory
        buf = torch.zeros(self.world, B, 2, dtype=torch.float32, device=val.device)
        buf[self.rank, :, 0] = val
        buf[self.rank, :, 1] = idx.to(torch.float32)
        if self.ar is not None:
            # an all-gather as an exact fp32 sum of disjoint slots, one-shot kernel
            self.ar(buf, out=buf, bits=16, algo="one_shot")
        else:
            dist.all_reduce(buf, group=self.group)
        best = buf[:, :, 0].argmax(dim=0)  # first maximum = lowest rank
        return buf[best, torch.arange(B, device=val.device), 1].to(torch.int64)


# ------------------------------------------------------------------------------------------
# KV cache
# ------------------------------------------------------------------------------------------
@dataclass
class KVCache:
    """Paged KV cache of one rank: per layer [pages, kv_heads, page, head_dim]."""
    k: list
    v: list
    block_table: torch.Tensor  # [B, pages_per_seq] int32
    seq_lens: torch.Tensor     # [B] int32, tokens already in the cache
    page: int

    @staticmethod
    def allocate(n_layers: int, batch: int, max_len: int, nkv: int, hd: int, device, dtype=torch.bfloat16,
                 page: int = 64) -> "KVCache":
        pps = (max_len + page - 1) // page
        pages = batch * pps
        k = [torch.empty(pages, nkv, page, hd, device=device, dtype=dtype) for _ in range(n_layers)]
        v = [torch.empty(pages, nkv, page, hd, device=device, dtype=dtype) for _ in range(n_layers)]
        bt = torch.arange(pages, device=device, dtype=torch.int32).view(batch, pps)
        return KVCache(k, v, bt, torch.zeros(batch, device=device, dtype=torch.int32), page)

    @property
    def capacity(self) -> int:
        """Tokens per sequence the block table can hold."""
        return self.block_table.shape[1] * self.page

    def slots(self, b_idx: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
        """Cache slot of each (sequence, position); -1 (not cached) past the capacity, so a
        step past the end never indexes outside the block table."""
        pidx = (pos // self.page).to(torch.long).clamp(max=self.block_table.shape[1] - 1)
        pg = self.block_table[b_idx, pidx].to(torch.int64)
        slot = pg * self.page + (pos % self.page).to(torch.int64)
        return torch.where(pos < self.capacity, slot, torch.full_like(slot, -1))


# ------------------------------------------------------------------------------------------
# Modules (weights only; the forward is written against the fused buffers)
# ------------------------------------------------------------------------------------------
class _W(nn.Module):
    def __init__(self, w: torch.Tensor):
        super().__init__()
        self.weight = nn.Parameter(w, requires_grad=False)


class _Attn(nn.Module):
    def __init__(self, qkv: torch.Tensor, o: torch.Tensor, nq_rows: int, nkv_rows: int):
        super().__init__()
        self.register_buffer("qkv_fused", qkv, persistent=False)
        self.q_proj = _W(qkv[:nq_rows])
        self.k_proj = _W(qkv[nq_rows:nq_rows + nkv_rows])
        self.v_proj = _W(qkv[nq_rows + nkv_rows:])
        self.o_proj = _W(o)


class _MLP(nn.Module):
    def __init__(self, gate_up: torch.Tensor, down: torch.Tensor, inter: int):
        super().__init__()
        self.register_buffer("gate_up_fused", gate_up, persistent=False)
        self.gate_proj = _W(gate_up[:inter])
        self.up_proj = _W(gate_up[inter:])
        self.down_proj = _W(down)


class _Layer(nn.Module):
    def __init__(self, attn: _Attn, mlp: _MLP, ln1: torch.Tensor, ln2: torch.Tensor):
        super().__init__()
        self.self_attn = attn
        self.mlp = mlp
        self.input_layernorm = _W(ln1)
        self.post_attention_layernorm = _W(ln2)


class _Inner(nn.Module):
    def __init__(self, embed: torch.Tensor, layers, norm: torch.Tensor):
        super().__init__()
        self.embed_tokens = _W(embed)
        self.layers = nn.ModuleList(layers)
        self.norm = _W(norm)


class LlamaTP(nn.Module):
    """One rank's shard of a tensor-parallel Llama model (inference)."""

    def __init__(self, cfg: LlamaConfig | str, tp: Optional[TPContext] = None, device=None,
                 dtype: torch.dtype = torch.bfloat16, init: str = "shard", seed: int = 0, init_std: float = 0.02):
        """``init``: "shard" (random N(0, init_std) per rank), "full" (random full tensors
        from ``seed``, then this rank's slice: every TP degree gets the same model) or
        "empty" (uninitialised, for ``load_hf_state_dict`` / ``from_pretrained``)."""
        super().__init__()
        cfg = get_config(cfg) if isinstance(cfg, str) else cfg
        self.cfg = cfg
        self.tp = tp or TPContext(device=device)
        W, r = self.tp.world, self.tp.rank
        device = self.tp.device if device is None else torch.device(device)
        self.device = device
        self.dtype = dtype
        H, hd = cfg.hidden_size, cfg.head_dim
        assert cfg.num_heads % W == 0, "heads must divide by the TP degree"
        assert cfg.num_kv_heads % W == 0, "kv heads must divide by the TP degree"
        assert cfg.intermediate_size % W == 0, "intermediate size must divide by the TP degree"
        self.nq, self.nkv, self.hd = cfg.num_heads // W, cfg.num_kv_heads // W, hd
        self.inter = cfg.intermediate_size // W
        self.v_local = (cfg.vocab_size + W - 1) // W
        self.vocab_start = r * self.v_local

        def rnd(shape, full_shape=None, slicer=None, key=0):
            if init == "empty":  # weights come from a checkpoint (load_hf_state_dict)
                return torch.empty(shape, device=device, dtype=dtype)
            if init == "full":
                g = torch.Generator(device=device).manual_seed(seed * 1000003 + key)
                t = torch.empty(full_shape, device=device, dtype=dtype).normal_(0.0, init_std, generator=g)
                return slicer(t).contiguous()
            g = torch.Generator(device=device).manual_seed(seed * 1000003 + key * 131 + r)
            return torch.empty(shape, device=device, dtype=dtype).normal_(0.0, init_std, generator=g)

        nqr, nkvr = self.nq * hd, self.nkv * hd
        layers = []
        for i in range(cfg.num_layers):
            k0 = (i + 1) * 16
            q = rnd((nqr, H), (cfg.num_heads * hd, H), lambda t: t[r * nqr:(r + 1) * nqr], k0 + 1)
            k = rnd((nkvr, H), (cfg.num_kv_heads * hd, H), lambda t: t[r * nkvr:(r + 1) * nkvr], k0 + 2)
            v = rnd((nkvr, H), (cfg.num_kv_heads * hd, H), lambda t: t[r * nkvr:(r + 1) * nkvr], k0 + 3)
            qkv = torch.cat([q, k, v], 0).contiguous()
            del q, k, v
            o = rnd((H, nqr), (H, cfg.num_heads * hd), lambda t: t[:, r * nqr:(r + 1) * nqr], k0 + 4)
            I = self.inter
            gate = rnd((I, H), (cfg.intermediate_size, H), lambda t: t[r * I:(r + 1) * I], k0 + 5)
            up = rnd((I, H), (cfg.intermediate_size, H), lambda t: t[r * I:(r + 1) * I], k0 + 6)
            gu = torch.cat([gate, up], 0).contiguous()
            del gate, up
            down = rnd((H, I), (H, cfg.intermediate_size), lambda t: t[:, r * I:(r + 1) * I], k0 + 7)
            ones = torch.ones(H, device=device, dtype=dtype)
            layers.append(_Layer(_Attn(qkv, o, nqr, nkvr), _MLP(gu, down, I), ones.clone(), ones.clone()))
        emb = rnd((cfg.vocab_size, H), (cfg.vocab_size, H), lambda t: t, 1)
        self.model = _Inner(emb, layers, torch.ones(H, device=device, dtype=dtype))
        vpad = self.v_local * W
        head = rnd((self.v_local, H), (vpad, H), lambda t: t[r * self.v_local:(r + 1) * self.v_local], 2)
        if self.vocab_start + self.v_local > cfg.vocab_size:  # padded rows never win the argmax
            head[cfg.vocab_size - self.vocab_start:] = 0
        self.lm_head = _W(head)
        self.cos_sin = L.rope_cos_sin(cfg.max_position, hd, cfg.rope_theta, device, cfg.rope_scaling)
        self.timer = None  # utils.trace.OpTimer: per-operator device times of eager steps

    # --------------------------------------------------------------------------------------
    # ------------------------------------------------------------------ checkpoints
    # The reference loads Hugging Face weights with from_pretrained and slices the MLP in
    # memory (main.py:25-39, 190-194).  Here every decoder weight is sharded: rows of
    # q/k/v/gate/up (by head / by intermediate unit), columns of o_proj/down_proj, rows of
    # the vocab-parallel lm_head (padded to a multiple of the TP degree); the embedding and
    # the norms are replicated.
    def _split_dim(self, name: str) -> Optional[int]:
        if name == "lm_head.weight" or any(t in name for t in ("q_proj", "k_proj", "v_proj", "gate_proj", "up_proj")):
            return 0
        if "o_proj" in name or "down_proj" in name:
            return 1
        return None

    def _shard_of(self, name: str, full) -> torch.Tensor:
        """This rank's part of the full tensor ``full`` (a tensor or a safetensors slice)."""
        W, r = self.tp.world, self.tp.rank
        dim = self._split_dim(name)
        if dim is None or W == 1 and name != "lm_head.weight":
            return full[:] if not isinstance(full, torch.Tensor) else full
        if name == "lm_head.weight":
            lo = self.vocab_start
            hi = min(lo + self.v_local, self.cfg.vocab_size)
            part = full[lo:hi] if hi > lo else None
            out = torch.zeros(self.v_local, self.cfg.hidden_size, dtype=self.dtype)
            if part is not None:
                out[: hi - lo] = part.to(self.dtype)
            return out
        n = (full.shape[dim] if isinstance(full, torch.Tensor) else full.get_shape()[dim]) // W
        return full[r * n:(r + 1) * n] if dim == 0 else full[:, r * n:(r + 1) * n]

    @torch.no_grad()
    def load_hf_state_dict(self, sd, strict: bool = True) -> None:
        """Copy this rank's shard out of a full (unsharded) Hugging Face Llama state dict.

        ``sd`` maps HF names to full tensors (or lazily sliceable safetensors entries).  With
        ``tie_word_embeddings`` a missing ``lm_head.weight`` is taken from the embedding.
        """
        own = dict(self.named_parameters())
        missing = []
        for name, p in own.items():
            src_name = name
            if name not in sd and name == "lm_head.weight" and "model.embed_tokens.weight" in sd:
                src_name = "model.embed_tokens.weight"
            if src_name not in sd:
                missing.append(name)
                continue
            part = self._shard_of(name, sd[src_name])
            if tuple(part.shape) != tuple(p.shape):
                raise ValueError(f"{name}: checkpoint shard {tuple(part.shape)} != parameter {tuple(p.shape)}")
            p.data.copy_(part.to(device=p.device, dtype=p.dtype))
        if strict and missing:
            raise KeyError(f"checkpoint lacks {missing[:4]}{' ...' if len(missing) > 4 else ''}")

    @torch.no_grad()
    def full_state_dict(self) -> "dict[str, torch.Tensor]":
        """The unsharded Hugging Face state dict, gathered from every rank (on every rank,
        on the CPU).  Collective: all ranks of the group must call it."""
        W = self.tp.world
        out = {}
        for name, p in self.named_parameters():
            dim = self._split_dim(name)
            t = p.detach()
            if W > 1 and dim is not None:
                parts = [torch.empty_like(t) for _ in range(W)]
                dist.all_gather(parts, t.contiguous(), group=self.tp.group)
                t = torch.cat(parts, dim)
            if name == "lm_head.weight":
                t = t[: self.cfg.vocab_size]
            out[name] = t.cpu().clone()
        return out

    def save_pretrained(self, path: str) -> None:
        """Write a Hugging Face style checkpoint (config.json + model.safetensors) of the full
        model from rank 0.  Collective (gathers the shards)."""
        import json
        import os
        from safetensors.torch import save_file
        full = self.full_state_dict()
        if self.tp.rank == 0:
            os.makedirs(path, exist_ok=True)
            if self.cfg.tie_word_embeddings:
                full.pop("lm_head.weight", None)
            save_file({k: v.contiguous() for k, v in full.items()}, os.path.join(path, "model.safetensors"))
            with open(os.path.join(path, "config.json"), "w") as f:
                json.dump(self.cfg.to_hf_dict(), f, indent=1)
        if self.tp.world > 1:
            dist.barrier(group=self.tp.group)

    @classmethod
    def from_pretrained(cls, path: str, tp: Optional[TPContext] = None, device=None,
                        dtype: torch.dtype = torch.bfloat16) -> "LlamaTP":
        """Build this rank's shard from a Hugging Face Llama checkpoint directory
        (config.json + *.safetensors).  Each rank reads only its slices of the files."""
        import glob
        import json
        import os
        from safetensors import safe_open
        with open(os.path.join(path, "config.json")) as f:
            cfg = LlamaConfig.from_hf_dict(json.load(f), name=os.path.basename(os.path.normpath(path)))
        model = cls(cfg, tp, device, dtype=dtype, init="empty")
        files = sorted(glob.glob(os.path.join(path, "*.safetensors")))
        if not files:
            raise FileNotFoundError(f"no *.safetensors under {path}")
        handles = [safe_open(fn, framework="pt", device="cpu") for fn in files]
        index = {}
        for h in handles:
            for k in h.keys():
                index[k] = h
        lazy = {k: index[k].get_slice(k) for k in index}
        model.load_hf_state_dict(lazy)
        return model

    def new_cache(self, batch: int, max_len: int, page: int = 64) -> KVCache:
        return KVCache.allocate(self.cfg.num_layers, batch, max_len, self.nkv, self.hd, self.device, self.dtype, page)

    def _layer(self, li: int, h: torch.Tensor, x: torch.Tensor, attn_fn, pos, slots, cache: Optional[KVCache],
               sp: bool = False):
        """One decoder layer.  h: residual stream [M, H] (updated in place; with ``sp`` only
        this rank's row shard [R, H]); x: its norm [M, H].

        Returns the input norm of the next layer (or the final norm after the last one).
        """
        cfg, tp = self.cfg, self.tp
        lay = self.model.layers[li]
        eps = cfg.rms_eps
        t = self.timer
        kc = cache.k[li] if cache is not None else None
        vc = cache.v[li] if cache is not None else None
        if pos is not None and self.hd == 128 and x.shape[0] > 64:
            # prefill: RoPE and the KV-cache write run in the qkv GEMM's epilogue
            with maybe_region(t, "qkv_gemm+rope_kv"):
                qkv = G.linear_qkv_rope(x, lay.self_attn.qkv_fused, pos, self.cos_sin, self.nq, self.nkv, kc, vc,
                                        slots)
        else:
            with maybe_region(t, "qkv_gemm"):
                qkv = G.linear(x, lay.self_attn.qkv_fused)
            with maybe_region(t, "rope_kv"):
                if pos is None:  # decode: position seq_lens - 1 and the cache slot, in the kernel
                    L.rope_kv_decode(qkv, self.cos_sin, self.nq, self.nkv, self.hd, kc, vc, cache.block_table,
                                     cache.seq_lens)
                else:
                    L.rope_kv(qkv, pos, self.cos_sin, self.nq, self.nkv, self.hd, kc, vc, slots)
        with maybe_region(t, "attention"):
            o = attn_fn(qkv, li)
        if sp:
            with maybe_region(t, "o_proj_gemm+allreduce+norm"):
                x = tp.linear_all_reduce_norm(o, lay.self_attn.o_proj.weight, h, lay.post_attention_layernorm.weight,
                                              eps)
        elif tp.world == 1:
            with maybe_region(t, "o_proj_gemm"):
                G.linear_residual(o, lay.self_attn.o_proj.weight, h, out=h)
            with maybe_region(t, "rmsnorm"):
                x = L.rmsnorm(h, lay.post_attention_layernorm.weight, eps)
        else:
            with maybe_region(t, "o_proj_gemm+allreduce"):
                ar = tp.linear_all_reduce(o, lay.self_attn.o_proj.weight)
            with maybe_region(t, "rmsnorm"):
                x = L.rmsnorm(ar, lay.post_attention_layernorm.weight, eps, residual=h)
        with maybe_region(t, "gate_up_gemm_swiglu"):
            act = G.linear_swiglu(x, lay.mlp.gate_up_fused)
        nxt = (self.model.layers[li + 1].input_layernorm.weight if li + 1 < cfg.num_layers else self.model.norm.weight)
        if sp:
            with maybe_region(t, "down_gemm+allreduce+norm"):
                return tp.linear_all_reduce_norm(act, lay.mlp.down_proj.weight, h, nxt, eps)
        if tp.world == 1:
            with maybe_region(t, "down_gemm"):
                G.linear_residual(act, lay.mlp.down_proj.weight, h, out=h)
            with maybe_region(t, "rmsnorm"):
                return L.rmsnorm(h, nxt, eps)
        with maybe_region(t, "down_gemm+allreduce"):
            ar = tp.linear_all_reduce(act, lay.mlp.down_proj.weight)
        with maybe_region(t, "rmsnorm"):
            return L.rmsnorm(ar, nxt, eps, residual=h)

    def _head(self, x_last: torch.Tensor, sampler: Optional[Sampler] = None) -> torch.Tensor:
        """Next token per row: greedy, or drawn by ``sampler`` (the same on every rank)."""
        logits = G.linear(x_last, self.lm_head.weight)
        valid = max(0, min(self.v_local, self.cfg.vocab_size - self.vocab_start))  # padded rows never count
        if sampler is not None and sampler.top_p < 1.0:
            full = self.tp.gather_vocab(logits)[:, : self.cfg.vocab_size]
            return sampler.full(full)
        if sampler is not None:
            val, idx = sampler.local(logits, self.vocab_start, valid)
        else:
            val, idx = L.argmax(logits, self.vocab_start, valid=valid)
        return self.tp.gather_argmax(val, idx)

    @torch.no_grad()
    def loss(self, ids: torch.Tensor) -> torch.Tensor:
        """Mean next-token negative log-likelihood of ``ids [B, S]`` (perplexity = exp(loss)).

        The lm_head is vocab-parallel, so the softmax statistics are combined across ranks
        (max, sum of exponentials, target logit) with three small all-reduces.
        """
        B, S = ids.shape
        x = self._hidden(ids, None)                              # [B*S, H], final norm applied
        logits = G.linear(x, self.lm_head.weight).float()        # [B*S, V_local]
        vs, vl = self.vocab_start, self.v_local
        valid = min(vl, self.cfg.vocab_size - vs)
        logits[:, valid:] = float("-inf")
        tgt = ids[:, 1:].reshape(-1)
        lg = logits.view(B, S, -1)[:, :-1].reshape(B * (S - 1), -1)
        m = lg.max(dim=-1).values
        if self.tp.world > 1:
            dist.all_reduce(m, op=dist.ReduceOp.MAX, group=self.tp.group)
        se = (lg - m[:, None]).exp().sum(-1)
        local = (tgt >= vs) & (tgt < vs + valid)
        t_logit = torch.where(local, lg.gather(1, (tgt - vs).clamp(0, vl - 1)[:, None]).squeeze(1),
                              torch.zeros_like(m))
        if self.tp.world > 1:
            dist.all_reduce(se, group=self.tp.group)
            dist.all_reduce(t_logit, group=self.tp.group)
        return (se.log() + m - t_logit).mean()

    def _hidden(self, ids: torch.Tensor, cache: Optional[KVCache]) -> torch.Tensor:
        B, S = ids.shape
        h = L.embedding(ids.reshape(-1), self.model.embed_tokens.weight)
        pos = torch.arange(S, device=self.device, dtype=torch.int64).repeat(B)
        slots = None
        if cache is not None:
            slots = cache.slots(torch.arange(B, device=self.device).repeat_interleave(S), pos)
        x = L.rmsnorm(h, self.model.layers[0].input_layernorm.weight, self.cfg.rms_eps)
        sp = self.tp.sp_active(B * S, self.cfg.hidden_size)
        if sp:  # keep only this rank's rows of the residual stream
            R, lo, n = self.tp.sp_rows(B * S)
            shard = torch.zeros(R, self.cfg.hidden_size, device=h.device, dtype=h.dtype)
            shard[:n] = h[lo:lo + n]
            h = shard

        def attn(qkv, li):
            return A.prefill_attention(qkv, B, S, self.nq, self.nkv, self.hd)

        for li in range(self.cfg.num_layers):
            x = self._layer(li, h, x, attn, pos, slots, cache, sp=sp)
        if cache is not None:
            cache.seq_lens.fill_(S)
        return x

    @torch.no_grad()
    def prefill(self, ids: torch.Tensor, cache: Optional[KVCache] = None, return_last_hidden: bool = False,
                sampler: Optional[Sampler] = None):
        """Causal forward over ``ids [B, S]`` (int64, on device); returns the next tokens [B]
        (greedy, or drawn by ``sampler``).

        With ``cache``, k/v of all positions are written to it and ``seq_lens`` becomes S.
        """
        B, S = ids.shape
        x = self._hidden(ids, cache)
        x_last = x.view(B, S, -1)[:, -1].contiguous()
        nxt = self._head(x_last, sampler)
        if return_last_hidden:
            return nxt, x_last
        return nxt

    @torch.no_grad()
    def decode_step(self, tokens: torch.Tensor, cache: KVCache, sampler: Optional[Sampler] = None) -> torch.Tensor:
        """One token per sequence: appends to the cache and returns the next tokens [B]
        (greedy, or drawn by ``sampler``)."""
        cfg = self.cfg
        t = self.timer
        with maybe_region(t, "embedding+rmsnorm"):
            h = L.embedding(tokens.reshape(-1), self.model.embed_tokens.weight)
            x = L.rmsnorm(h, self.model.layers[0].input_layernorm.weight, cfg.rms_eps)
        cache.seq_lens.add_(1)
        nqr = self.nq * self.hd

        def attn(qkv, li):  # q is read in place from the fused qkv rows
            return A.decode_attention(qkv[:, :nqr], cache.k[li], cache.v[li], cache.block_table, cache.seq_lens,
                                      self.nq, self.nkv, self.hd)

        for li in range(cfg.num_layers):
            x = self._layer(li, h, x, attn, None, None, cache)
        with maybe_region(t, "lm_head+argmax"):
            return self._head(x, sampler)

    @torch.no_grad()
    def capture_prefill(self, batch: int, seq: int, cache: Optional[KVCache] = None,
                        warmup: int = 2) -> "GraphedStep":
        """Capture one prefill of ``[batch, seq]`` tokens as a CUDA graph.

        Every kernel of the step (GEMMs, attention, the fused all-reduces, the head) is
        replayed with one launch; all ranks of a tensor-parallel group must capture
        together.  Returns a callable taking token ids and returning next tokens.
        """
        cache = cache if cache is not None else self.new_cache(batch, seq)
        ids = torch.zeros(batch, seq, dtype=torch.int64, device=self.device)
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            for _ in range(warmup):
                self.prefill(ids, cache)
        torch.cuda.current_stream(self.device).wait_stream(side)
        torch.cuda.synchronize(self.device)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            out = self.prefill(ids, cache)
        return GraphedStep(graph, ids, out)

    @torch.no_grad()
    def capture_decode(self, cache: KVCache, warmup: int = 2, sampler: Optional[Sampler] = None) -> "GraphedStep":
        """Capture one decode step (one token per sequence) as a CUDA graph.

        The graph reads positions from ``cache.seq_lens`` on the device, so the same graph
        serves every step; the caller must not exceed the cache's capacity.  With
        ``sampler`` the step samples; its step counter lives on the device, so every replay
        draws fresh noise (the warm-up steps advance it too).
        """
        B = cache.seq_lens.numel()
        tok = torch.zeros(B, dtype=torch.int64, device=self.device)
        saved = cache.seq_lens.clone()
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            for _ in range(warmup):
                self.decode_step(tok, cache, sampler)
                cache.seq_lens.copy_(saved)
        torch.cuda.current_stream(self.device).wait_stream(side)
        torch.cuda.synchronize(self.device)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            out = self.decode_step(tok, cache, sampler)
        cache.seq_lens.copy_(saved)  # capture does not run the kernels, but keep state explicit
        return GraphedStep(graph, tok, out)

    @torch.no_grad()
    def generate(self, ids: torch.Tensor, max_new_tokens: int, cache: Optional[KVCache] = None,
                 do_sample: bool = False, temperature: float = 1.0, top_p: float = 1.0,
                 seed: Optional[int] = None, sampler: Optional[Sampler] = None, monitor=None,
                 check_every: int = 16) -> torch.Tensor:
        """Generate ``max_new_tokens`` tokens per sequence; returns them as [B, max_new_tokens].

        Greedy by default.  ``do_sample=True`` samples from softmax(logits / temperature),
        restricted to the top-p nucleus when ``top_p < 1`` (the knobs of Hugging Face
        ``generate``, which the reference calls with ``do_sample=True, temperature=0.7``).
        Every rank draws the same tokens: the seed is rank 0's (``seed`` or a random one),
        broadcast once.  Collective: all ranks of the group call it together.

        ``monitor`` (``utils.health.PeerMonitor``): before the prefill and every
        ``check_every`` decode steps the stream is synchronised and the peers' heartbeats
        checked, so that a lost rank raises ``PeerLostError`` on the host instead of the
        next step's collectives waiting out their device timeout.
        """
        def check():
            if monitor is not None:
                torch.cuda.current_stream(self.device).synchronize()
                monitor.check()

        if sampler is None and do_sample:
            sampler = Sampler(self.tp, temperature=temperature, top_p=top_p, seed=seed)
        B, S = ids.shape
        if cache is None:
            cache = self.new_cache(B, S + max_new_tokens)
        if S + max_new_tokens - 1 > cache.capacity:
            raise ValueError(f"cache holds {cache.capacity} tokens per sequence; {S} + {max_new_tokens} requested")
        out = torch.empty(B, max_new_tokens, dtype=torch.int64, device=self.device)
        check()
        tok = self.prefill(ids, cache, sampler=sampler)
        out[:, 0] = tok
        for t in range(1, max_new_tokens):
            if t % check_every == 0:
                check()
            tok = self.decode_step(tok, cache, sampler)
            out[:, t] = tok
        return out


class GraphedStep:
    """A captured model step: copy inputs into the static buffer, replay, read the output."""

    def __init__(self, graph, inp: torch.Tensor, out: torch.Tensor):
        self.graph = graph
        self.inp = inp
        self.out = out

    def __call__(self, x: Optional[torch.Tensor] = None) -> torch.Tensor:
        if x is not None:
            self.inp.copy_(x.view_as(self.inp), non_blocking=True)
        self.graph.replay()
        return self.out

    def release(self):
        self.graph.reset()


def smoke_forward(device) -> None:
    """One tiny prefill + decode step of the flagship architecture (random weights).

    GQA (8 query / 2 kv heads) and 4 x 64 prompt tokens, so the step runs the CTA-pair
    GEMMs (256 rows), the tcgen05 prefill attention, the split-K GEMMs and the tensor-core
    decode attention."""
    from .config import LlamaConfig
    cfg = LlamaConfig("smoke", 1024, 2048, 1, 8, 2, 1024, head_dim=128, max_position=512)
    m = LlamaTP(cfg, device=device)
    ids = torch.randint(0, cfg.vocab_size, (4, 64), device=device)
    cache = m.new_cache(4, 80)
    tok = m.prefill(ids, cache)
    tok2 = m.decode_step(tok, cache)
    torch.cuda.synchronize(device)
    assert tok.shape == (4,) and tok2.shape == (4,)
    assert G.gemm_status() == 0
