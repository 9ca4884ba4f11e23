"""The benchmark workloads (the five configurations the cuda target is measured on), as torch modules + seeded
synthetic data, the way the reference freezes its contract model (anvil/model.py:151-300,
anvil/codesign/workloads.py:40-80).

The torch modules are a nanoGPT-shaped family written here: pre-LN blocks (LayerNorm -> causal multi-head
attention -> residual -> LayerNorm -> 4x MLP with GELU -> residual), biases, learned token + position embeddings
and a tied LM head. Weights are N(0, 0.02) (biases zero, LayerNorm weight 1 / bias 0) from torch.manual_seed(seed).
No public dataset or checkpoint is involved: inputs are numpy default_rng(seed) draws of the stated shapes.

    c1  one block, n_embd 32, 2 heads, T 8, batch 1, 16 calibration inputs x ~ N(0, 1)          (seed 0)
    c2  2-layer model, vocab 64, block 16, n_embd 64, 4 heads, 32 calibration sequences, B 256   (seed 1)
    c3  GPT-2-small block, n_embd 768, 12 heads, MLP 3072, T 1024, B 64, 8 calibration batches  (seed 2)
    c4  int8 GEMM + requant sweep, M in {1024, 8192, 65536}, K = N in {768, 3072, 4096}           (seed 3)
    c5  12-layer GPT-2-small model, vocab 50304, T 1024, B 512, prefill                          (seed 4)
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np


@dataclass(frozen=True)
class GPTConfig:
    vocab_size: int = 50304
    block_size: int = 1024
    n_layer: int = 12
    n_head: int = 12
    n_embd: int = 768
    bias: bool = True


def _torch_modules():
    import torch
    import torch.nn as nn
    import torch.nn.functional as F

    class CausalSelfAttention(nn.Module):
        def __init__(self, cfg: GPTConfig):
            super().__init__()
            self.c_attn = nn.Linear(cfg.n_embd, 3 * cfg.n_embd, bias=cfg.bias)
            self.c_proj = nn.Linear(cfg.n_embd, cfg.n_embd, bias=cfg.bias)
            self.n_head = cfg.n_head

        def forward(self, x):
            B, T, C = x.size()
            q, k, v = self.c_attn(x).split(C, dim=2)
            hd = C // self.n_head
            q = q.view(B, T, self.n_head, hd).transpose(1, 2)
            k = k.view(B, T, self.n_head, hd).transpose(1, 2)
            v = v.view(B, T, self.n_head, hd).transpose(1, 2)
            y = F.scaled_dot_product_attention(q, k, v, is_causal=True)
            y = y.transpose(1, 2).contiguous().view(B, T, C)
            return self.c_proj(y)

    class MLP(nn.Module):
        def __init__(self, cfg: GPTConfig):
            super().__init__()
            self.c_fc = nn.Linear(cfg.n_embd, 4 * cfg.n_embd, bias=cfg.bias)
            self.gelu = nn.GELU()
            self.c_proj = nn.Linear(4 * cfg.n_embd, cfg.n_embd, bias=cfg.bias)

        def forward(self, x):
            return self.c_proj(self.gelu(self.c_fc(x)))

    class Block(nn.Module):
        def __init__(self, cfg: GPTConfig):
            super().__init__()
            self.ln_1 = nn.LayerNorm(cfg.n_embd, bias=cfg.bias)
            self.attn = CausalSelfAttention(cfg)
            self.ln_2 = nn.LayerNorm(cfg.n_embd, bias=cfg.bias)
            self.mlp = MLP(cfg)

        def forward(self, x):
            x = x + self.attn(self.ln_1(x))
            return x + self.mlp(self.ln_2(x))

    class GPT(nn.Module):
        def __init__(self, cfg: GPTConfig):
            super().__init__()
            self.cfg = cfg
            self.wte = nn.Embedding(cfg.vocab_size, cfg.n_embd)
            self.wpe = nn.Embedding(cfg.block_size, cfg.n_embd)
            self.h = nn.ModuleList([Block(cfg) for _ in range(cfg.n_layer)])
            self.ln_f = nn.LayerNorm(cfg.n_embd, bias=cfg.bias)
            self.lm_head = nn.Linear(cfg.n_embd, cfg.vocab_size, bias=False)
            self.wte.weight = self.lm_head.weight           # tied

        def forward(self, idx):
            T = idx.size(1)
            pos = torch.arange(0, T, dtype=torch.long, device=idx.device)
            x = self.wte(idx) + self.wpe(pos)
            for blk in self.h:
                x = blk(x)
            return self.lm_head(self.ln_f(x))

    def init_(m):
        for mod in m.modules():
            if isinstance(mod, nn.Linear):
                nn.init.normal_(mod.weight, 0.0, 0.02)
                if mod.bias is not None:
                    nn.init.zeros_(mod.bias)
            elif isinstance(mod, nn.Embedding):
                nn.init.normal_(mod.weight, 0.0, 0.02)
        return m

    return Block, GPT, init_


def build_block(cfg: GPTConfig, seed: int):
    import torch
    Block, _, init_ = _torch_modules()
    torch.manual_seed(seed)
    return init_(Block(cfg)).eval()


def build_gpt(cfg: GPTConfig, seed: int):
    import torch
    _, GPT, init_ = _torch_modules()
    torch.manual_seed(seed)
    return init_(GPT(cfg)).eval()


@dataclass(frozen=True)
class Config:
    name: str
    kind: str                     # "block" | "model" | "gemm"
    cfg: GPTConfig | None
    seq: int                      # T
    batch: int                    # evaluation batch
    n_calib: int                  # calibration samples
    seed: int


CONFIGS = {
    "c1": Config("c1", "block", GPTConfig(vocab_size=1, block_size=8, n_layer=1, n_head=2, n_embd=32), 8, 1, 16, 0),
    "c2": Config("c2", "model", GPTConfig(vocab_size=64, block_size=16, n_layer=2, n_head=4, n_embd=64), 16, 256,
                 32, 1),
    "c3": Config("c3", "block", GPTConfig(vocab_size=1, block_size=1024, n_layer=1, n_head=12, n_embd=768), 1024, 64,
                 8, 2),
    "c5": Config("c5", "model", GPTConfig(), 1024, 512, 4, 4),
}
GEMM_SWEEP = [(m, k, k) for m in (1024, 8192, 65536) for k in (768, 3072, 4096)]      # (M, K, N), config c4


def module_and_data(name: str, batch: int | None = None, calib: int | None = None):
    """(torch module, example input, calibration inputs, evaluation-input generator) of a config.
    The generator draws `n` evaluation inputs from default_rng(seed + 1000)."""
    import torch
    c = CONFIGS[name]
    rng = np.random.default_rng(c.seed)
    ncal = c.n_calib if calib is None else calib
    if c.kind == "block":
        mod = build_block(c.cfg, c.seed)
        cal = rng.standard_normal((ncal, c.seq, c.cfg.n_embd))
        ex = torch.zeros((1, c.seq, c.cfg.n_embd))

        def gen(n, rng=np.random.default_rng(c.seed + 1000)):
            return rng.standard_normal((n, c.seq, c.cfg.n_embd))
    else:
        mod = build_gpt(c.cfg, c.seed)
        cal = rng.integers(0, c.cfg.vocab_size, (ncal, c.seq))
        ex = torch.zeros((1, c.seq), dtype=torch.long)

        def gen(n, rng=np.random.default_rng(c.seed + 1000)):
            return rng.integers(0, c.cfg.vocab_size, (n, c.seq))
    return mod, ex, cal, gen


def compile_config(name: str, params=None, calib: int | None = None):
    """anvil.compile of a config's torch module on its calibration data -> (CompiledModel, input generator)."""
    from .driver import compile as _compile
    mod, ex, cal, gen = module_and_data(name, calib=calib)
    cm = _compile(mod, (ex,), [cal], params)
    return cm, gen


def gemm_case(m, k, n, seed=3):
    """Config c4 operands: A[M, K], B[K, N] ~ U[-127, 127] int8 and (M, s) = fixed_point([m], [K 127^2]) with the
    real multiplier m ~ U[2^-12, 2^-6]."""
    from .frontend.numerics import fixed_point
    rng = np.random.default_rng(seed)
    a = rng.integers(-127, 128, (m, k), dtype=np.int8)
    b = rng.integers(-127, 128, (k, n), dtype=np.int8)
    (mult,), s = fixed_point([float(rng.uniform(2 ** -12, 2 ** -6))], [k * 127 * 127])
    return a, b, mult, s


def tokens_per_step(name: str, batch: int | None = None) -> int:
    c = CONFIGS[name]
    return (batch or c.batch) * c.seq


def algorithmic_ops(name: str, batch: int | None = None) -> dict:
    """Integer ops of one forward: GEMMs 2MNK, attention 4 hd T(T+1)/2 per (sequence, head) (kept entries)."""
    c = CONFIGS[name]
    B, T, C, L = (batch or c.batch), c.seq, c.cfg.n_embd, c.cfg.n_layer
    nh = c.cfg.n_head
    hd = C // nh
    gemm = 2 * B * T * (3 * C * C + C * C + 8 * C * C) * L
    if c.kind == "model":
        gemm += 2 * B * T * C * c.cfg.vocab_size
    attn = 4 * hd * T * (T + 1) // 2 * nh * B * L
    return {"gemm": gemm, "attention": attn, "total": gemm + attn}
