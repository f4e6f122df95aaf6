"""The synthetic MoE decoder of BASELINE configs[4], run through the C-ABI.

48 layers, hidden 2048, GQA 32 query / 4 KV heads of dim 128 with NeoX RoPE
(theta 1e6), RMSNorm (eps 1e-6, weights 1), an MoE FFN per layer (128
experts, top-8 softmax routing, expert FFN 768, SwiGLU), vocab 151936; every
matmul weight NVFP4 (random init), the router f32 N(0, 0.02), an f16 KV cache.
T sequences decode one token each per step.  A step is, per layer:

    rmsnorm -> QKV matvec (NVFP4 x q8_1) -> RoPE + f16 KV append ->
    GQA decode attention (tcgen05) -> O matvec + residual -> rmsnorm ->
    MoE layer (router top-k, expert grouping, expert matvecs, slot-order
    combine) + residual

then rmsnorm -> LM head matvec -> arg-max -> the next step's embedding rows.
The step's position lives on the device, so the whole step is captured once
as a CUDA graph and replayed: a prompt of P tokens is fed by P replays (the
embedding kernel reads the prompt while pos < P), then every replay decodes
one token per sequence.  This is the decode loop llama.cpp runs around the
reference's hot path (its ROUTE -> MOEFFN and LMHEAD windows,
src/fr_win_flint_sm120.cu:1602-2409 and :1176-1282); the runner itself is a
benchmark and test harness, not a serving stack.
"""
from __future__ import annotations

import ctypes as C

from . import (_ptr, _stream, call, gemv_f32, gemv_tiled, lib, moe_ffn, moe_ffn_tiled, row_bytes, tile_experts,
               tile_nvfp4)


class Config:
    def __init__(self, n_layers=48, hidden=2048, n_head=32, n_kv=4, head_dim=128, n_expert=128, n_used=8,
                 n_ff=768, vocab=151936, ctx=2048, rope_base=1e6, eps=1e-6):
        self.n_layers, self.hidden, self.n_head, self.n_kv, self.head_dim = n_layers, hidden, n_head, n_kv, head_dim
        self.n_expert, self.n_used, self.n_ff, self.vocab, self.ctx = n_expert, n_used, n_ff, vocab, ctx
        self.rope_base, self.eps = rope_base, eps

    @property
    def qkv_width(self):
        return (self.n_head + 2 * self.n_kv) * self.head_dim


class MoeDecoder:
    """Weights generated on the device (seeded), buffers for `batch`
    sequences.  `dense` chooses the layout of the attention and LM-head
    matrices ("ggml": in place; "tiled": repacked once for the FP4 tensor-core
    matvec); `experts` the expert layout ("ggml": dp4a expert matvecs;
    "tiled": FP4 tensor-core expert matvecs)."""

    def __init__(self, cfg: Config, batch: int, seed: int = 0x5EED5000, dense: str = "ggml",
                 experts: str = "ggml", device=None):
        import torch
        self.cfg, self.T = cfg, batch
        self.dev = device or torch.device("cuda", torch.cuda.current_device())
        self.dense, self.experts = dense, experts
        c, dev = cfg, self.dev
        H, L = c.hidden, c.n_layers
        s = torch.cuda.current_stream()

        def nvfp4(seed_, rows, K):
            w = torch.empty((rows, row_bytes(K)), dtype=torch.uint8, device=dev)
            call("fr_synth_nvfp4_device", seed_, rows, K, 0.05, _ptr(w), _stream(s))
            return w

        g = torch.Generator(device=dev)
        self.layers = []
        for li in range(L):
            b = seed + 1000 * li
            lay = {"wqkv": nvfp4(b + 1, c.qkv_width, H), "wo": nvfp4(b + 2, H, c.n_head * c.head_dim)}
            g.manual_seed(b + 3)
            lay["wr"] = torch.randn((c.n_expert, H), generator=g, device=dev, dtype=torch.float32) * 0.02
            lay["wg"] = nvfp4(b + 4, c.n_expert * c.n_ff, H)
            lay["wu"] = nvfp4(b + 5, c.n_expert * c.n_ff, H)
            lay["wd"] = nvfp4(b + 6, c.n_expert * H, c.n_ff)
            if dense == "tiled":
                lay["wqkv"] = tile_nvfp4(lay["wqkv"], c.qkv_width, H)
                lay["wo"] = tile_nvfp4(lay["wo"], H, c.n_head * c.head_dim)
            if experts == "tiled":
                lay["wg"] = tile_experts(lay["wg"], c.n_expert, c.n_ff, H)
                lay["wu"] = tile_experts(lay["wu"], c.n_expert, c.n_ff, H)
                lay["wd"] = tile_experts(lay["wd"], c.n_expert, H, c.n_ff)
            self.layers.append(lay)
        self.embed = nvfp4(seed + 7, c.vocab, H)
        self.lm_head = nvfp4(seed + 8, c.vocab, H)
        if dense == "tiled":
            self.lm_head = tile_nvfp4(self.lm_head, c.vocab, H)
        self.norm_w = torch.ones(H, dtype=torch.float32, device=dev)     # every RMSNorm weight is 1
        T = batch
        kv_shape = (L, T, c.n_kv, c.ctx, c.head_dim)
        self.kc = torch.zeros(kv_shape, dtype=torch.float16, device=dev)
        self.vc = torch.zeros(kv_shape, dtype=torch.float16, device=dev)
        f = dict(dtype=torch.float32, device=dev)
        self.x = [torch.zeros((T, H), **f), torch.zeros((T, H), **f)]
        self.xn = torch.zeros((T, H), **f)
        self.qkv = torch.zeros((T, c.qkv_width), **f)
        self.q_r = torch.zeros((T, c.n_head, c.head_dim), **f)
        self.attn = torch.zeros((T, c.n_head * c.head_dim), **f)
        self.logits = torch.zeros((T, c.vocab), **f)
        self.tok = torch.zeros(T, dtype=torch.int32, device=dev)
        self.pos = torch.zeros(1, dtype=torch.int32, device=dev)
        self.prompt = None
        self.prompt_len = 0
        torch.cuda.synchronize()

    # ------------------------------------------------------------ the step
    def set_prompt(self, prompt_tokens):
        """prompt_tokens: int32 [T, P] on the device; resets the position."""
        self.prompt = prompt_tokens.contiguous()
        self.prompt_len = int(prompt_tokens.shape[1])
        self.pos.zero_()

    def _matvec(self, w, x, N, K, out, resid=None, stream=None):
        if self.dense == "tiled":
            return gemv_tiled(w, N, K, x=x, resid=resid, out=out, stream=stream)
        return gemv_f32(w, x, N, K, resid=resid, out=out, stream=stream)

    def step(self, stream=None):
        """One decode step of every sequence (capturable)."""
        c, T, st = self.cfg, self.T, _stream(stream)
        H = c.hidden
        x, x2 = self.x
        plen = self.prompt_len
        call("fr_embed_nvfp4", _ptr(self.embed), c.vocab, H, _ptr(self.prompt) if plen else None, plen, plen,
             _ptr(self.tok), _ptr(self.pos), _ptr(x), T, st)
        for li, lay in enumerate(self.layers):
            call("fr_rmsnorm_f32", _ptr(x), _ptr(self.norm_w), _ptr(self.xn), T, H, C.c_float(c.eps), st)
            self._matvec(lay["wqkv"], self.xn, c.qkv_width, H, self.qkv, stream=stream)
            call("fr_rope_kv_f16", _ptr(self.qkv), _ptr(self.pos), _ptr(self.q_r), _ptr(self.kc[li]),
                 _ptr(self.vc[li]), T, c.n_head, c.n_kv, c.head_dim, c.ctx, C.c_float(c.rope_base), st)
            call("fr_attn_decode_f16", _ptr(self.q_r), _ptr(self.kc[li]), _ptr(self.vc[li]), _ptr(self.pos),
                 _ptr(self.attn), T, c.n_head, c.n_kv, c.head_dim, c.ctx, st)
            self._matvec(lay["wo"], self.attn, H, c.n_head * c.head_dim, x2, resid=x, stream=stream)
            call("fr_rmsnorm_f32", _ptr(x2), _ptr(self.norm_w), _ptr(self.xn), T, H, C.c_float(c.eps), st)
            moe = moe_ffn_tiled if self.experts == "tiled" else moe_ffn
            moe(self.xn, lay["wr"], lay["wg"], lay["wu"], lay["wd"], H, c.n_ff, c.n_expert, c.n_used, resid=x2,
                out=x, stream=stream)
        call("fr_rmsnorm_f32", _ptr(x), _ptr(self.norm_w), _ptr(self.xn), T, H, C.c_float(c.eps), st)
        self._matvec(self.lm_head, self.xn, c.vocab, H, self.logits, stream=stream)
        call("fr_argmax_f32", _ptr(self.logits), T, c.vocab, _ptr(self.tok), st)
        call("fr_pos_advance", _ptr(self.pos), st)

    def weight_bytes(self):
        """NVFP4 weight bytes a T=1 step reads at most (all experts count)."""
        c = self.cfg
        per_layer = (row_bytes(c.hidden) * (c.qkv_width + 3 * c.n_expert * c.n_ff) +
                     row_bytes(c.n_head * c.head_dim) * c.hidden + c.n_expert * c.hidden * 4)
        return c.n_layers * per_layer + 2 * row_bytes(c.hidden) * c.vocab


def attention_flops(cfg: Config, T: int, n_keys: int) -> float:
    return 4.0 * T * cfg.n_head * cfg.head_dim * n_keys

