"""Synthetic training workloads of the benchmark configurations.

The models are the reference demos' architectures (examples/demo_15_mini_gpt.py
MiniGPT / Block / CausalSelfAttention / SparseFFN, examples/demo_05_mnist.py
MLP) sized per the benchmark configs, with every sparse projection a
``SparseLinear``.  Data is synthetic (seeded uniform token ids / N(0,1)
features): the reference's datasets are not needed to measure the path.

  cfg2  MLP 784->512->10 (ReLU), both 90% sparse, batch 256, SGD 0.1,
        SET every 100 steps (drop 0.3)
  cfg4  char transformer d384 x6 layers, 6 heads, ctx 256, vocab 65,
        attention 70% / FFN 90% sparse, batch 64, AdamW 3e-4, RigL / 100
  cfg5  byte-level mini-GPT d768 x8 layers, 12 heads, ctx 512, vocab 256,
        attention 70% / FFN 90% sparse, batch 32 per GPU, AdamW 3e-4,
        SET every 200 steps
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

from .nn import SparseLinear, sparse_mlp


@dataclass(frozen=True)
class GPTConfig:
    name: str
    d_model: int
    n_layers: int
    n_heads: int
    seq_len: int
    vocab: int
    d_ff: int
    attn_sparsity: float
    ffn_sparsity: float
    batch: int
    lr: float
    router: str
    update_freq: int
    drop_fraction: float = 0.3


CFG4 = GPTConfig("cfg4-char-transformer-10M", 384, 6, 6, 256, 65, 1536, 0.7, 0.9, 64, 3e-4,
                 "RigL", 100)
CFG5 = GPTConfig("cfg5-byte-mini-gpt-60M", 768, 8, 12, 512, 256, 3072, 0.7, 0.9, 32, 3e-4,
                 "SET", 200)


def _sparse_linear(device):
    def make(fin, fout, sparsity):
        return SparseLinear(fin, fout, bias=False, sparsity=sparsity, device=device)
    return make


class CausalSelfAttention(nn.Module):
    def __init__(self, d_model, n_heads, attn_sparsity, linear):
        super().__init__()
        self.n_heads = n_heads
        self.d_head = d_model // n_heads
        self.qkv = linear(d_model, 3 * d_model, attn_sparsity)
        self.o = linear(d_model, d_model, attn_sparsity)

    def forward(self, x):
        B, T, C = x.shape
        q, k, v = self.qkv(x).chunk(3, dim=-1)
        q = q.view(B, T, self.n_heads, self.d_head).transpose(1, 2)
        k = k.view(B, T, self.n_heads, self.d_head).transpose(1, 2)
        v = v.view(B, T, self.n_heads, self.d_head).transpose(1, 2)
        att = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        return self.o(att.transpose(1, 2).contiguous().view(B, T, C))


class SparseFFN(nn.Module):
    def __init__(self, d_model, d_ff, sparsity, linear):
        super().__init__()
        self.fc_up = linear(d_model, d_ff, sparsity)
        self.fc_down = linear(d_ff, d_model, sparsity)

    def forward(self, x):
        if isinstance(self.fc_up, SparseLinear) and isinstance(self.fc_down, SparseLinear):
            return sparse_mlp(x, self.fc_up, self.fc_down, "gelu")
        return self.fc_down(F.gelu(self.fc_up(x)))


class Block(nn.Module):
    def __init__(self, cfg: GPTConfig, linear):
        super().__init__()
        self.ln1 = nn.LayerNorm(cfg.d_model)
        self.attn = CausalSelfAttention(cfg.d_model, cfg.n_heads, cfg.attn_sparsity, linear)
        self.ln2 = nn.LayerNorm(cfg.d_model)
        self.ffn = SparseFFN(cfg.d_model, cfg.d_ff, cfg.ffn_sparsity, linear)

    def forward(self, x):
        x = x + self.attn(self.ln1(x))
        return x + self.ffn(self.ln2(x))


class MiniGPT(nn.Module):
    """Decoder-only transformer; dense embeddings / LayerNorms / head, sparse
    attention projections and FFN.  ``linear(in, out, sparsity)`` builds each
    sparse projection (default: SparseLinear on ``device``); all parameters
    are drawn from torch's CPU generator in construction order and the dense
    parts are then placed on ``device``."""

    def __init__(self, cfg: GPTConfig, device=None, linear=None):
        super().__init__()
        self.cfg = cfg
        dev = torch.device(device) if device is not None else None
        if linear is None:
            linear = _sparse_linear(device)
            if dev is None:
                dev = torch.device("cuda", torch.cuda.current_device())
        dev = dev or torch.device("cpu")
        self.tok_emb = nn.Embedding(cfg.vocab, cfg.d_model)
        self.pos_emb = nn.Embedding(cfg.seq_len, cfg.d_model)
        self.blocks = nn.ModuleList([Block(cfg, linear) for _ in range(cfg.n_layers)])
        self.ln_f = nn.LayerNorm(cfg.d_model)
        self.head = nn.Linear(cfg.d_model, cfg.vocab, bias=False)
        self.register_buffer("pos_ids", torch.arange(cfg.seq_len))
        for mod in [self.tok_emb, self.pos_emb, self.ln_f, self.head]:
            mod.to(dev)
        for b in self.blocks:
            b.ln1.to(dev)
            b.ln2.to(dev)
        self.pos_ids = self.pos_ids.to(dev)

    def forward(self, idx):
        B, T = idx.shape
        x = self.tok_emb(idx) + self.pos_emb(self.pos_ids[:T])
        for blk in self.blocks:
            x = blk(x)
        return self.head(self.ln_f(x))


def make_mlp(device=None) -> nn.Sequential:  # noqa: D401
    """cfg2 MLP: SparseLinear(784,512) -> ReLU -> SparseLinear(512,10)."""
    return nn.Sequential(SparseLinear(784, 512, sparsity=0.9, device=device), nn.ReLU(),
                         SparseLinear(512, 10, sparsity=0.9, device=device))


def synthetic_tokens(cfg: GPTConfig, batch: int, seed: int) -> torch.Tensor:
    """Uniform-random token ids [batch, seq_len + 1] (inputs + shifted targets)."""
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, cfg.vocab, (batch, cfg.seq_len + 1), generator=g)


def lm_loss(model: MiniGPT, tokens: torch.Tensor) -> torch.Tensor:
    x, y = tokens[:, :-1], tokens[:, 1:]
    logits = model(x)
    return F.cross_entropy(logits.reshape(-1, logits.size(-1)), y.reshape(-1))


def sparse_live_weights(model: nn.Module) -> int:
    return sum(m.nnz for m in model.modules() if isinstance(m, SparseLinear))
