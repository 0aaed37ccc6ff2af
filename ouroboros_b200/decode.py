"""End-to-end decode of a BitNet b1.58 2B-class model around the ternary path.

The layer follows the reference's run_layer (cluster/src/infer/mod.rs:298-336):

    a  = rmsnorm(x, attn_norm)
    q, k, v = W_q a, W_k a, W_v a                      (ternary, this library)
    rope_neox(q, k) at the token's position (ops.rs:21-33)
    append k, v to the layer's KV cache; causal GQA attention (mod.rs:337-)
    o  = W_o rmsnorm(attn, attn_sub_norm)              (ternary)
    h1 = x + o
    f  = rmsnorm(h1, ffn_norm)
    s  = rmsnorm(silu(W_gate f) * (W_up f), ffn_sub_norm)   (ternary gate/up)
    x' = h1 + W_down s                                  (ternary)

then the output norm and the tied embedding as the lm_head (an F16 weight),
greedy next token (finite_argmax, fused into the lm_head launch). Configuration defaults of ArchConfig (mod.rs:45-55): hidden 2560,
20 heads / 5 KV heads of 128, FFN 6912, eps 1e-5, RoPE base 500000.

Every ternary projection runs through the C ABI (the path this library
rebuilds). The ops around it run either as this library's fused kernels
(`fused=True`, the default: each RMSNorm -- with the residual add, or the
SiLU·up product of the FFN sub-norm -- fused into the projection group that
reads it, ouroq_gemm_norm_f32act; RoPE + KV append + split-sequence GQA
attention in one launch, ouroq_rope_attention_decode) or as plain torch operations
(`fused=False`, the unfused host path kept as a cross-check). fp32 throughout
like the reference, KV cache included. A
decode step has static shapes -- the position lives in a device tensor -- so it
is captured as one CUDA graph. Weights are random (synthetic).
"""
from __future__ import annotations

import math

HIDDEN, FFN, N_HEAD, N_KV, HEAD_DIM = 2560, 6912, 20, 5, 128
EPS, ROPE_BASE = 1e-5, 500000.0


class Decoder:
    def __init__(self, ctx, *, layers=30, batch=1, context=1024, generate=256, vocab=128256,
                 device=None, seed=0, lm_head=True, fused=True):
        import torch
        import ouroboros_b200 as oq
        self.torch, self.oq, self.ctx = torch, oq, ctx
        self.L, self.B, self.vocab = layers, batch, vocab
        self.tmax = context + generate
        self.context = context
        self.lm_head = lm_head
        self.fused = fused
        dev = device or torch.device("cuda", ctx.device)
        self.dev = dev
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        self.gen = g

        def tern(M, K):
            r = torch.randint(0, 4, (M, K), generator=g, device=dev, dtype=torch.uint8)
            codes = (r == 3).to(torch.uint8) * 2 + ((r == 1) | (r == 2)).to(torch.uint8)
            c = codes.view(M, K // 4, 4)
            packed = (c[..., 0] | (c[..., 1] << 2) | (c[..., 2] << 4) | (c[..., 3] << 6)).contiguous()
            nz = torch.count_nonzero(codes != 1).item()
            return ctx.upload_device(oq.TERNARY2, packed, M, K, None, 0.02 * nz / (M * K))

        def gain(n):
            return 1.0 + 0.02 * torch.randn(n, generator=g, device=dev)

        self.layers = []
        for _ in range(layers):
            self.layers.append({
                "q": tern(HIDDEN, HIDDEN), "k": tern(N_KV * HEAD_DIM, HIDDEN),
                "v": tern(N_KV * HEAD_DIM, HIDDEN), "o": tern(HIDDEN, HIDDEN),
                "gate": tern(FFN, HIDDEN), "up": tern(FFN, HIDDEN), "down": tern(HIDDEN, FFN),
                "attn_norm": gain(HIDDEN), "attn_sub_norm": gain(HIDDEN),
                "ffn_norm": gain(HIDDEN), "ffn_sub_norm": gain(FFN),
            })
        self.tok_embd = (0.02 * torch.randn((vocab, HIDDEN), generator=g, device=dev)).half()
        # the tied lm_head: token_embd as an F16 weight (the shard's dtype 1)
        self.head = ctx.upload_device(oq.F16, self.tok_embd, vocab, HIDDEN)
        self.output_norm = gain(HIDDEN)
        B, T = batch, self.tmax
        # KV cache [layer][B, kv_head, T, dim], the first `context` positions filled
        self.kc = torch.zeros((layers, B, N_KV, T, HEAD_DIM), device=dev)
        self.vc = torch.zeros((layers, B, N_KV, T, HEAD_DIM), device=dev)
        self.kc[:, :, :, :context].normal_(generator=g)
        self.vc[:, :, :, :context].normal_(generator=g)
        self.pos = torch.full((1,), context, dtype=torch.long, device=dev)
        self.tokens = torch.randint(0, vocab, (B,), generator=g, device=dev)
        # RoPE tables (neox: rotate halves), indexed by position on the device
        half = HEAD_DIM // 2
        inv = ROPE_BASE ** (-torch.arange(half, device=dev, dtype=torch.float64) * 2 / HEAD_DIM)
        ang = torch.arange(T, device=dev, dtype=torch.float64)[:, None] * inv[None, :]
        self.cos, self.sin = ang.cos().float(), ang.sin().float()
        self.steps = torch.arange(T, device=dev)
        # persistent work buffers (the graph reads and writes the same memory)
        f32 = dict(dtype=torch.float32, device=dev)
        self.buf = {n: torch.empty((B, m), **f32) for n, m in
                    [("q", HIDDEN), ("k", N_KV * HEAD_DIM), ("v", N_KV * HEAD_DIM),
                     ("o", HIDDEN), ("gate", FFN), ("up", FFN), ("down", HIDDEN),
                     ("x", HIDDEN), ("h1", HIDDEN), ("a", HIDDEN), ("attn", HIDDEN),
                     ("b", HIDDEN), ("f", HIDDEN), ("s", FFN)]}
        self.q8 = {k: torch.empty((B, k), dtype=torch.int8, device=dev) for k in (HIDDEN, FFN)}
        self.s8 = {k: torch.empty((B,), **f32) for k in (HIDDEN, FFN)}
        self.stream = torch.cuda.Stream(device=dev)
        # the fills above ran on the current stream; the step runs on self.stream
        self.stream.wait_stream(torch.cuda.current_stream(dev))

    # ---- the ternary path (this library) ----
    def tern(self, names, layer, x):
        """y_n = W_n x for the projections `names` of one layer, all reading x."""
        ws = [layer[n] for n in names]
        ys = [self.buf[n] for n in names]
        if self.B <= self.oq_fused_max():
            self.ctx.gemm_group_f32act(ws, [x] * len(ws), ys, stream=self.stream)
        else:
            K = x.shape[1]
            q, s = self.q8[K], self.s8[K]
            self.ctx.quantize_act(x, q=q, s_x=s, stream=self.stream)
            for w, y in zip(ws, ys):
                self.ctx.gemm(w, q, s, y=y, stream=self.stream)
        return ys

    def oq_fused_max(self):
        return 8  # grouped fp32-activation calls take up to 8 tokens

    # ---- host path around it ----
    def rmsnorm(self, x, w):
        t = self.torch
        return x * t.rsqrt(x.pow(2).mean(-1, keepdim=True) + EPS) * w

    def rope(self, v, heads):
        # v [B, heads*128] -> [B, heads, 128], rotate halves at position pos
        t = self.torch
        v = v.view(self.B, heads, HEAD_DIM)
        c = self.cos.index_select(0, self.pos)[:, None, :]
        s = self.sin.index_select(0, self.pos)[:, None, :]
        a, b = v[..., :HEAD_DIM // 2], v[..., HEAD_DIM // 2:]
        return t.cat([a * c - b * s, b * c + a * s], dim=-1)

    def layer(self, li, x):
        t = self.torch
        L = self.layers[li]
        a = self.rmsnorm(x, L["attn_norm"])
        q, k, v = self.tern(("q", "k", "v"), L, a)
        q = self.rope(q, N_HEAD)
        k = self.rope(k, N_KV)
        self.kc[li].index_copy_(2, self.pos, k[:, :, None, :])
        self.vc[li].index_copy_(2, self.pos, v.view(self.B, N_KV, 1, HEAD_DIM))
        mask = (self.steps <= self.pos)[None, None, None, :]
        attn = t.nn.functional.scaled_dot_product_attention(
            q[:, :, None, :], self.kc[li], self.vc[li], attn_mask=mask, enable_gqa=True)
        attn = attn.reshape(self.B, HIDDEN)
        (o,) = self.tern(("o",), L, self.rmsnorm(attn, L["attn_sub_norm"]))
        h1 = x + o
        f = self.rmsnorm(h1, L["ffn_norm"])
        gate, up = self.tern(("gate", "up"), L, f)
        s = self.rmsnorm(t.nn.functional.silu(gate) * up, L["ffn_sub_norm"])
        (d,) = self.tern(("down",), L, s)
        return h1 + d

    def layer_fused(self, li, first):
        """One layer on the library's kernels, each norm fused into the
        projection group that reads it. On entry buf x holds the hidden state
        (first layer) or h1 / down of the previous layer hold its two residual
        terms, added inside the first launch."""
        c, bf, L = self.ctx, self.buf, self.layers[li]
        st = self.stream
        qkv = [L[n] for n in ("q", "k", "v")]
        out_qkv = [bf["q"], bf["k"], bf["v"]]
        if first:
            c.gemm_norm_f32act(qkv, bf["x"], L["attn_norm"], out_qkv, eps=EPS, stream=st)
        else:
            c.gemm_norm_f32act(qkv, bf["h1"], L["attn_norm"], out_qkv, residual=bf["down"],
                               h=bf["x"], eps=EPS, stream=st)
        c.rope_attention_decode(bf["q"], bf["k"], bf["v"], self.kc[li], self.vc[li], self.pos,
                                N_HEAD, N_KV, ROPE_BASE, out=bf["attn"], stream=st)
        c.gemm_norm_f32act([L["o"]], bf["attn"], L["attn_sub_norm"], [bf["o"]], eps=EPS, stream=st)
        c.gemm_norm_f32act([L["gate"], L["up"]], bf["x"], L["ffn_norm"], [bf["gate"], bf["up"]],
                           residual=bf["o"], h=bf["h1"], eps=EPS, stream=st)
        c.gemm_norm_f32act([L["down"]], bf["gate"], L["ffn_sub_norm"], [bf["down"]],
                           residual=bf["up"], swiglu=True, eps=EPS, stream=st)

    def step(self):
        """One token for every sequence: embed, 30 layers, lm_head, greedy pick."""
        t = self.torch
        x = self.tok_embd.index_select(0, self.tokens).float()
        if self.fused:
            self.buf["x"].copy_(x)
            for li in range(self.L):
                self.layer_fused(li, li == 0)
            xo = self.buf["x"]  # the final residual sum
            h = self.ctx.rmsnorm(self.buf["h1"], self.output_norm, y=self.buf["a"],
                                 residual=self.buf["down"], h=xo, stream=self.stream)
            x = xo
        else:
            for li in range(self.L):
                x = self.layer(li, x)
            h = self.rmsnorm(x, self.output_norm)
        if self.lm_head:
            # tied lm_head + finite_argmax in one launch (mod.rs:190-194)
            self.ctx.argmax_token(self.head, h, tokens=self.tokens, stream=self.stream)
        self.pos.add_(1)
        return x

    def ternary_only_step(self):
        """The same ternary calls on static inputs (for the time share)."""
        x = self.buf["o"]
        f = self.buf["down"]
        for L in self.layers:
            self.tern(("q", "k", "v"), L, x)
            self.tern(("o",), L, x)
            self.tern(("gate", "up"), L, x)
            self.tern(("down",), L, self.buf["gate"])
        return f

    def capture(self, fn):
        """A CUDA graph of fn (one step). The warm-up steps it runs first are
        undone: position and next tokens are put back, and the cache entries
        they wrote lie past the position, where the next step overwrites them
        before attention reads them."""
        t = self.torch
        tok0 = self.tokens.clone()
        with t.cuda.stream(self.stream):
            fn()
            # one eager step inside an NVTX range named after fn, for profilers
            with t.cuda.nvtx.range(fn.__name__):
                fn()
            self.pos.fill_(self.context)
        self.stream.synchronize()
        g = t.cuda.CUDAGraph()
        with t.cuda.graph(g, stream=self.stream):
            fn()
        self.pos.fill_(self.context)
        self.tokens.copy_(tok0)
        t.cuda.synchronize()
        return g

    def free(self):
        for L in self.layers:
            for n in ("q", "k", "v", "o", "gate", "up", "down"):
                L[n].free()
        self.head.free()
