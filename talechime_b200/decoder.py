"""Q8_0 decoder (the decode and batched-prefill benchmark workloads: the VoxCPM BaseLM-style Llama decoder):
batch-1 decode steps and a batched prompt pass (``prefill``).

Per layer (crates/voxcpm/src/transformer.rs:107-155): rms_norm -> fused q|k|v Q8_0 linear
-> RoPE on q and k, k and v appended to the f32 KV cache -> attention over the cache ->
o linear -> residual add -> rms_norm -> fused gate|up Q8_0 linear -> SwiGLU -> down
linear -> residual add; then the final rms_norm, the Q8_0 LM head and the greedy
argmax.  Every operation is a libq8lin kernel (by default with the norms, SwiGLU and
residual adds fused into the projections); the position and the current token live
in device memory, so ``step()`` is capture-safe and one captured CUDA graph replays for
every decode step (``q8lin_argmax`` writes the next token and advances the position).

Weights are GGUF Q8_0 block arrays (bytes / numpy / torch uint8) and f32 norm vectors;
q|k|v and gate|up are stored as fused weights (rows q, then k, then v; gate, then up).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Optional

import numpy as np
import torch

from . import _lib
from ._lib import check
from .qmatmul import QMatMul, _stream_ptr
from .tp_mlp import swiglu


@dataclass(frozen=True)
class DecoderConfig:
    hidden: int = 2048
    layers: int = 28
    heads: int = 16
    kv_heads: int = 16
    head_dim: int = 128
    inter: int = 6144
    vocab: int = 73448
    max_t: int = 640
    eps: float = 1e-5
    rope_theta: float = 10000.0

    @property
    def qkv_rows(self) -> int:
        return (self.heads + 2 * self.kv_heads) * self.head_dim


def rope_tables(cfg: DecoderConfig, factors: Optional[np.ndarray] = None) -> tuple[np.ndarray, np.ndarray]:
    """cos/sin [max_t][head_dim/2] as transformer.rs:48-60 builds them: freq_i =
    theta^(-2i/d) in f64 rounded to f32, divided by the factors (f32), angle = pos * freq
    (f32), then f32 cos/sin."""
    half = cfg.head_dim // 2
    freq = np.array([cfg.rope_theta ** (-(2 * i) / cfg.head_dim) for i in range(half)], dtype=np.float64)
    f = freq.astype(np.float32)
    if factors is not None:
        f = (f / np.asarray(factors, dtype=np.float32)).astype(np.float32)
    pos = np.arange(cfg.max_t, dtype=np.float32)[:, None]
    ang = (pos * f[None, :]).astype(np.float32)
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


# GGUF metadata the reference checks before loading the BaseLM (crates/voxcpm/src/model.rs:119-133).
VOXCPM_BASELM_EXPECT = {"embedding_length": 2048, "block_count": 28, "feed_forward_length": 6144,
                        "vocab_size": 73448, "attention.head_count": 16, "attention.head_count_kv": 2,
                        "attention.key_length": 128, "attention.value_length": 128}


def config_from_gguf(g, max_t: int = 640, arch: Optional[str] = None) -> DecoderConfig:
    """DecoderConfig from a GGUF file's `{arch}.*` metadata (general.architecture when
    `arch` is None); eps and RoPE theta are the reference's constants
    (transformer.rs:49-51,104)."""
    arch = arch or g.value("general.architecture")
    u = lambda name: g.to_u32(f"{arch}.{name}")
    heads = u("attention.head_count")
    hidden = u("embedding_length")
    return DecoderConfig(hidden=hidden, layers=u("block_count"), heads=heads,
                         kv_heads=u("attention.head_count_kv"), head_dim=u("attention.key_length"),
                         inter=u("feed_forward_length"), vocab=u("vocab_size"), max_t=max_t)


def weights_from_gguf(g, cfg: DecoderConfig, prefix: str = "") -> tuple[dict, Optional[np.ndarray]]:
    """The decoder's weight dict from GGUF tensors with the reference's names
    (transformer.rs:78-88: {prefix}blk.{i}.attn_norm / attn_q / attn_k / attn_v /
    attn_output / ffn_norm / ffn_gate / ffn_up / ffn_down; model.rs:135-141:
    token_embd, output_norm, rope_factors_short).  q|k|v and gate|up are fused by
    concatenating their Q8_0 block rows (no re-quantization); the LM head is
    `output.weight`, or the embedding when the file ties them.  Returns (weights,
    rope_factors or None)."""
    def blocks(name, rows, k):
        b = g.q8_0_blocks(name)
        if b.shape != (rows, k // 32 * 34):
            raise _lib.Q8LinError(_lib.ERR_SHAPE, f"tensor '{name}' is {b.shape[0]} x {b.shape[1] // 34 * 32}, "
                                                  f"expected {rows} x {k}")
        return b

    H, D = cfg.hidden, cfg.head_dim
    layers = []
    for i in range(cfg.layers):
        p = f"{prefix}blk.{i}"
        layers.append({
            "attn_norm": g.tensor(f"{p}.attn_norm.weight").reshape(-1),
            "qkv": np.concatenate([blocks(f"{p}.attn_q.weight", cfg.heads * D, H),
                                   blocks(f"{p}.attn_k.weight", cfg.kv_heads * D, H),
                                   blocks(f"{p}.attn_v.weight", cfg.kv_heads * D, H)]),
            "o": blocks(f"{p}.attn_output.weight", H, cfg.heads * D),
            "ffn_norm": g.tensor(f"{p}.ffn_norm.weight").reshape(-1),
            "gate_up": np.concatenate([blocks(f"{p}.ffn_gate.weight", cfg.inter, H),
                                       blocks(f"{p}.ffn_up.weight", cfg.inter, H)]),
            "down": blocks(f"{p}.ffn_down.weight", H, cfg.inter),
        })
    embd = blocks("token_embd.weight", cfg.vocab, H)
    head = blocks("output.weight", cfg.vocab, H) if "output.weight" in g else embd
    factors = g.tensor("rope_factors_short.weight").reshape(-1) if "rope_factors_short.weight" in g else None
    return {"token_embd": embd, "output": head, "output_norm": g.tensor("output_norm.weight").reshape(-1),
            "layers": layers}, factors


class Q8Decoder:
    """Weights, KV cache and step buffers of one decoder on one GPU."""

    @classmethod
    def from_gguf(cls, path: str, device: torch.device | int | str = 0, max_t: int = 640,
                  expect: Optional[dict] = None, arch: Optional[str] = None) -> "Q8Decoder":
        """Load a decoder from a GGUF file (Model::load_files_with_cancel's BaseLM half,
        crates/voxcpm/src/model.rs:118-145).  `expect` maps `{arch}.`-relative metadata
        keys to required u32 values (VOXCPM_BASELM_EXPECT for the production file)."""
        from .gguf import GGUFFile

        with GGUFFile(path) as g:
            arch = arch or g.value("general.architecture")
            for name, val in (expect or {}).items():
                g.expect_u32(f"{arch}.{name}", val)
            cfg = config_from_gguf(g, max_t=max_t, arch=arch)
            weights, factors = weights_from_gguf(g, cfg)
        return cls(cfg, weights, device=device, rope_factors=factors)

    def __init__(self, cfg: DecoderConfig, weights: dict, device: torch.device | int | str = 0,
                 rope_factors: Optional[np.ndarray] = None, batch: int = 1):
        """`batch` sequences share the weights and the position; each has its own KV cache
        (prefill() takes [batch, T] tokens); the decode step serves batch 1."""
        if batch < 1:
            raise ValueError("batch must be positive")
        self.batch = int(batch)
        if cfg.head_dim != 128:
            raise _lib.Q8LinError(_lib.ERR_SHAPE, "the decode attention kernel takes head_dim 128")
        self.cfg = cfg
        dev = torch.device("cuda", device) if isinstance(device, int) else torch.device(device)
        if dev.type != "cuda":
            raise ValueError("the decoder runs on a CUDA device; there is no CPU path")
        if dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        self.device = dev
        H = cfg.hidden

        def mat(blocks, n, k):
            return QMatMul.from_gguf_blocks(blocks, n, k, device=dev)

        def vec(v):
            t = torch.as_tensor(np.asarray(v, dtype=np.float32) if not isinstance(v, torch.Tensor) else v)
            return t.to(dev, dtype=torch.float32).contiguous()

        self.embed = mat(weights["token_embd"], cfg.vocab, H)
        self.lm_head = mat(weights["output"], cfg.vocab, H)
        self.out_norm = vec(weights["output_norm"])
        self.layers = []
        for li in range(cfg.layers):
            w = weights["layers"][li]
            self.layers.append({
                "attn_norm": vec(w["attn_norm"]),
                "qkv": mat(w["qkv"], cfg.qkv_rows, H),
                "o": mat(w["o"], H, cfg.heads * cfg.head_dim),
                "ffn_norm": vec(w["ffn_norm"]),
                "gate_up": mat(w["gate_up"], 2 * cfg.inter, H),
                "down": mat(w["down"], H, cfg.inter),
            })
        cos, sin = rope_tables(cfg, rope_factors)
        self.cos = torch.from_numpy(cos).to(dev)
        self.sin = torch.from_numpy(sin).to(dev)
        kv_shape = (cfg.kv_heads, cfg.max_t, cfg.head_dim)
        if self.batch > 1:
            kv_shape = (self.batch,) + kv_shape
        self.k_cache = [torch.zeros(kv_shape, device=dev) for _ in range(cfg.layers)]
        self.v_cache = [torch.zeros(kv_shape, device=dev) for _ in range(cfg.layers)]
        f = lambda n: torch.zeros(n, device=dev)
        self.x, self.h = f(H), f(H)
        self.qkv, self.q = f(cfg.qkv_rows), f(cfg.heads * cfg.head_dim)
        self.attn, self.o_out, self.d_out = f(cfg.heads * cfg.head_dim), f(H), f(H)
        self.gu, self.logits = f(2 * cfg.inter), f(cfg.vocab)
        self.hmid = f(cfg.inter)  # silu(gate) * up of the persistent step
        self.token = torch.zeros(1, dtype=torch.int32, device=dev)
        self.pos = torch.zeros(1, dtype=torch.int32, device=dev)
        L = _lib.lib()
        self.attn_ws = torch.zeros(L.q8lin_attention_workspace_size(cfg.heads, cfg.max_t), dtype=torch.uint8,
                                   device=dev)
        self.argmax_ws = torch.zeros(L.q8lin_argmax_workspace_size(), dtype=torch.uint8, device=dev)

    @staticmethod
    def _p(t: torch.Tensor) -> ctypes.c_void_p:
        return ctypes.c_void_p(t.data_ptr())

    def reset(self, token: int = 0) -> None:
        """Empty the cache (position 0) and set the current token."""
        self.pos.zero_()
        self.token.fill_(int(token))

    MODES = ("persistent", "fused", "unfused")

    def step(self, mode: str = "fused") -> None:
        """One decode step for the token at self.token / position self.pos; afterwards
        self.token holds the greedy next token, self.logits its logits, pos advanced.

        mode "persistent": the whole step is one cooperative launch of the persistent
        decode-step kernel (q8lin_step_run), weights streamed ahead of the data;
        "fused": one launch per operation with rms_norm and SwiGLU inside the following
        projection's activation quantization, the residual adds inside the o / down
        projections and RoPE + KV append inside the attention kernel (5 launches per
        layer); "unfused": 11 launches per layer, one per reference operation."""
        if self.batch != 1:
            raise ValueError("the decode step serves batch 1; this decoder holds "
                             f"{self.batch} sequences (prefill only)")
        if mode == "persistent":
            check(_lib.lib().q8lin_step_run(self._persistent(), ctypes.c_void_p(_stream_ptr(self.device))))
        elif mode == "fused":
            self._step_fused()
        elif mode == "unfused":
            self._step_unfused()
        else:
            raise ValueError(f"mode must be one of {self.MODES}")

    def _persistent(self) -> ctypes.c_void_p:
        """The decode step as a q8lin_step program (built once, then reused)."""
        if getattr(self, "_step_handle", None) is not None:
            return self._step_handle
        cfg, L, P = self.cfg, _lib.lib(), lambda t: t.data_ptr()
        ops = [_lib.Op(kind=_lib.OP_EMBED, weight=self.embed.handle.value, y=P(self.x))]
        for li, w in enumerate(self.layers):
            ops.append(_lib.Op(kind=_lib.OP_GEMV, prologue=_lib.PROLOGUE_RMSNORM, weight=w["qkv"].handle.value,
                               x=P(self.x), y=P(self.qkv), norm_weight=P(w["attn_norm"]), eps=cfg.eps))
            ops.append(_lib.Op(kind=_lib.OP_ATTENTION, x=P(self.qkv), y=P(self.attn), k_cache=P(self.k_cache[li]),
                               v_cache=P(self.v_cache[li]), cos_t=P(self.cos), sin_t=P(self.sin), hq=cfg.heads,
                               hkv=cfg.kv_heads, head_dim=cfg.head_dim, max_t=cfg.max_t))
            ops.append(_lib.Op(kind=_lib.OP_GEMV, weight=w["o"].handle.value, x=P(self.attn), y=P(self.x),
                               residual=P(self.x)))
            ops.append(_lib.Op(kind=_lib.OP_GEMV, prologue=_lib.PROLOGUE_RMSNORM, epilogue=_lib.EPILOGUE_SWIGLU,
                               weight=w["gate_up"].handle.value, x=P(self.x), y=P(self.hmid),
                               norm_weight=P(w["ffn_norm"]), eps=cfg.eps))
            ops.append(_lib.Op(kind=_lib.OP_GEMV, weight=w["down"].handle.value, x=P(self.hmid), y=P(self.x),
                               residual=P(self.x)))
        ops.append(_lib.Op(kind=_lib.OP_GEMV, prologue=_lib.PROLOGUE_RMSNORM, weight=self.lm_head.handle.value,
                           x=P(self.x), y=P(self.logits), norm_weight=P(self.out_norm), eps=cfg.eps, argmax=1))
        ops.append(_lib.Op(kind=_lib.OP_ARGMAX))
        arr = (_lib.Op * len(ops))(*ops)
        h = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            check(L.q8lin_step_create(arr, len(ops), ctypes.c_void_p(P(self.pos)), ctypes.c_void_p(P(self.token)),
                                      self.device.index, ctypes.byref(h)))
        self._step_handle = h
        return h

    def __del__(self):
        h = getattr(self, "_step_handle", None)
        if h is not None and h.value:
            try:
                _lib.lib().q8lin_step_destroy(h)
            except Exception:
                pass
            self._step_handle = None

    def _step_fused(self) -> None:
        cfg, L, P = self.cfg, _lib.lib(), self._p
        s = ctypes.c_void_p(_stream_ptr(self.device))
        check(L.q8lin_embed_rows(self.embed.handle, P(self.token), 1, P(self.x), s))
        for li, w in enumerate(self.layers):
            w["qkv"].forward_fused(self.x, self.qkv, QMatMul.PROLOGUE_RMSNORM, w["attn_norm"], cfg.eps)
            # the step starts with the embedding launch after the previous step's argmax,
            # so the position and the cached rows are ready before this launch's wait
            check(L.q8lin_rope_attention_decode_ex(P(self.qkv), P(self.pos), P(self.cos), P(self.sin),
                                                   P(self.k_cache[li]), P(self.v_cache[li]), cfg.heads, cfg.kv_heads,
                                                   cfg.head_dim, cfg.max_t, P(self.attn), 1, s))
            w["o"].forward_fused(self.attn, self.x, residual=self.x)
            w["gate_up"].forward_fused(self.x, self.gu, QMatMul.PROLOGUE_RMSNORM, w["ffn_norm"], cfg.eps)
            w["down"].forward_fused(self.gu, self.x, QMatMul.PROLOGUE_SWIGLU, residual=self.x)
        self.lm_head.forward_fused(self.x, self.logits, QMatMul.PROLOGUE_RMSNORM, self.out_norm, cfg.eps)
        check(L.q8lin_argmax(P(self.logits), cfg.vocab, P(self.argmax_ws), self.argmax_ws.numel(), P(self.token),
                             P(self.pos), s))

    def _step_unfused(self) -> None:
        cfg, L, P = self.cfg, _lib.lib(), self._p
        s = ctypes.c_void_p(_stream_ptr(self.device))
        H = cfg.hidden
        check(L.q8lin_embed_rows(self.embed.handle, P(self.token), 1, P(self.x), s))
        for li, w in enumerate(self.layers):
            check(L.q8lin_rmsnorm(P(self.x), P(w["attn_norm"]), 1, H, cfg.eps, P(self.h), s))
            w["qkv"].forward(self.h.view(1, H), out=self.qkv.view(1, -1))
            check(L.q8lin_rope_kv(P(self.qkv), P(self.pos), P(self.cos), P(self.sin), P(self.k_cache[li]),
                                  P(self.v_cache[li]), cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.max_t,
                                  P(self.q), s))
            check(L.q8lin_attention_decode(P(self.q), P(self.k_cache[li]), P(self.v_cache[li]), P(self.pos),
                                           cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.max_t, P(self.attn_ws),
                                           self.attn_ws.numel(), P(self.attn), s))
            w["o"].forward(self.attn.view(1, -1), out=self.o_out.view(1, H))
            check(L.q8lin_add(P(self.x), P(self.o_out), H, s))
            check(L.q8lin_rmsnorm(P(self.x), P(w["ffn_norm"]), 1, H, cfg.eps, P(self.h), s))
            w["gate_up"].forward(self.h.view(1, H), out=self.gu.view(1, -1))
            w["down"].forward(swiglu(self.gu.view(1, -1), cfg.inter), out=self.d_out.view(1, H))
            check(L.q8lin_add(P(self.x), P(self.d_out), H, s))
        check(L.q8lin_rmsnorm(P(self.x), P(self.out_norm), 1, H, cfg.eps, P(self.h), s))
        self.lm_head.forward(self.h.view(1, H), out=self.logits.view(1, -1))
        check(L.q8lin_argmax(P(self.logits), cfg.vocab, P(self.argmax_ws), self.argmax_ws.numel(), P(self.token),
                             P(self.pos), s))

    def prefill(self, tokens) -> torch.Tensor:
        """Run a prompt as ONE batched forward: `tokens` [T] (batch 1) or [batch, T] ids at
        positions pos .. pos + T - 1 of every sequence (crates/voxcpm/src/model.rs:492-495,
        transformer.rs:107-155 with offset = pos): the linears at M = batch * T, RoPE and
        the KV append per row (q8lin_rope_kv_rows), causal attention (q8lin_attention_
        prefill), each residual add fused with the norm after it (q8lin_add_rmsnorm), then
        the final norm, LM head and greedy pick on each sequence's last row.  Returns the next token of each sequence (int32 [batch] on the device);
        afterwards the caches hold the T new rows, pos has advanced by T, self.logits
        holds the last row's logits (batch 1; self.prefill_logits [batch, vocab]) and,
        for batch 1, self.token the next token -- the state T decode steps over the same
        tokens leave.  Raises Q8LinError(ERR_SHAPE) past max_t, as the reference's
        "Transformer context limit exceeded" (transformer.rs:110-113)."""
        cfg, L, P = self.cfg, _lib.lib(), self._p
        tok = torch.as_tensor(np.asarray(tokens.cpu() if isinstance(tokens, torch.Tensor) else tokens),
                              dtype=torch.int32)
        if tok.dim() == 1:
            tok = tok.unsqueeze(0)
        if tok.dim() != 2 or tok.shape[0] != self.batch:
            raise _lib.Q8LinError(_lib.ERR_SHAPE, f"tokens must be [T] or [{self.batch}, T]; got {tuple(tok.shape)}")
        B, T = tok.shape
        pos0 = int(self.pos.item())
        if T == 0:
            raise _lib.Q8LinError(_lib.ERR_SHAPE, "prefill needs at least one token")
        if pos0 + T > cfg.max_t:
            raise _lib.Q8LinError(_lib.ERR_SHAPE, "Transformer context limit exceeded")
        return self._prefill_launches(tok.reshape(-1).to(self.device), B, T, pos0)

    def _prefill_launches(self, tok_d: torch.Tensor, B: int, T: int, pos0: int) -> torch.Tensor:
        """The device work of ``prefill`` for `tok_d` (int32 [B * T] on the device) at a
        host-known position pos0 (checked by the caller): kernel launches on the current
        stream and tensor allocations only, no host synchronisation."""
        cfg, L, P = self.cfg, _lib.lib(), self._p
        dev, H, M = self.device, cfg.hidden, B * T
        hd = cfg.heads * cfg.head_dim
        s = ctypes.c_void_p(_stream_ptr(dev))
        e = lambda *shape: torch.empty(shape, dtype=torch.float32, device=dev)
        x, hn, qkv, q, att, t1 = e(M, H), e(M, H), e(M, cfg.qkv_rows), e(M, hd), e(M, hd), e(M, H)
        gu, hm = e(M, 2 * cfg.inter), e(M, cfg.inter)
        check(L.q8lin_embed_rows(self.embed.handle, P(tok_d), M, P(x), s))
        check(L.q8lin_rmsnorm(P(x), P(self.layers[0]["attn_norm"]), M, H, cfg.eps, P(hn), s))
        for li, w in enumerate(self.layers):
            w["qkv"].forward(hn, out=qkv)
            check(L.q8lin_rope_kv_rows(P(qkv), B, T, pos0, P(self.cos), P(self.sin), P(self.k_cache[li]),
                                       P(self.v_cache[li]), cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.max_t,
                                       P(q), s))
            check(L.q8lin_attention_prefill(P(q), P(self.k_cache[li]), P(self.v_cache[li]), B, T, pos0, cfg.heads,
                                            cfg.kv_heads, cfg.head_dim, cfg.max_t, P(att), s))
            w["o"].forward(att, out=t1)
            # residual add + the norm after it, one pass: x += o(att); hn = ffn_norm(x)
            check(L.q8lin_add_rmsnorm(P(x), P(t1), P(w["ffn_norm"]), M, H, cfg.eps, P(hn), s))
            w["gate_up"].forward(hn, out=gu)
            check(L.q8lin_swiglu(P(gu), M, cfg.inter, P(hm), s))
            w["down"].forward(hm, out=t1)
            if li + 1 < len(self.layers):  # x += down(h); hn = next layer's attn_norm(x)
                check(L.q8lin_add_rmsnorm(P(x), P(t1), P(self.layers[li + 1]["attn_norm"]), M, H, cfg.eps, P(hn), s))
            else:
                check(L.q8lin_add(P(x), P(t1), M * H, s))
        last = e(B, H)
        for b in range(B):  # each sequence's last row
            check(L.q8lin_rmsnorm(ctypes.c_void_p(x.data_ptr() + ((b * T + T - 1) * H) * 4), P(self.out_norm), 1, H,
                                  cfg.eps, ctypes.c_void_p(last.data_ptr() + b * H * 4), s))
        logits = e(B, cfg.vocab)
        self.lm_head.forward(last, out=logits)
        nxt = torch.empty(B, dtype=torch.int32, device=dev)
        for b in range(B):
            check(L.q8lin_argmax(ctypes.c_void_p(logits.data_ptr() + b * cfg.vocab * 4), cfg.vocab,
                                 P(self.argmax_ws), self.argmax_ws.numel(), ctypes.c_void_p(nxt.data_ptr() + 4 * b),
                                 None, s))
        self.pos.fill_(pos0 + T)
        self.prefill_logits = logits
        if B == 1:
            self.logits.copy_(logits[0])
            self.token.copy_(nxt)
        return nxt

    def launches_per_step(self, mode: str = "fused") -> int:
        if mode == "persistent":
            return 1
        fused = mode == "fused"
        return 1 + self.cfg.layers * (5 if fused else 11) + (2 if fused else 3)

    def weight_bytes_per_step(self) -> int:
        cfg = self.cfg
        per_layer = (cfg.qkv_rows + cfg.hidden + 2 * cfg.inter) * cfg.hidden + cfg.hidden * cfg.inter
        return (cfg.layers * per_layer + cfg.vocab * cfg.hidden) * 34 // 32


def synthetic_weights(cfg: DecoderConfig, seed: int = 0, device: Optional[torch.device] = None) -> dict:
    """Random-init Q8_0 weights with the benchmark's distributions (qs uniform in [-127, 127],
    d = |N(0, 0.02)| / 127 as f16; norm weights 1), numpy on the host or torch uint8 on
    `device` (for the 2 GB full-size model)."""
    def blocks(n, k):
        nb = k // 32
        if device is None:
            from . import synth
            return synth.q8_0_blocks(rng, n, k)
        b = torch.empty((n, nb, 34), dtype=torch.uint8, device=device)
        b[:, :, 2:] = torch.randint(-127, 128, (n, nb, 32), generator=gen, device=device,
                                    dtype=torch.int8).view(torch.uint8)
        d = (torch.randn((n, nb), generator=gen, device=device).abs() * (0.02 / 127.0)).half()
        b[:, :, :2] = d.view(torch.uint8).view(n, nb, 2)
        return b

    rng = np.random.default_rng(seed)
    gen = None
    if device is not None:
        gen = torch.Generator(device=device)
        gen.manual_seed(seed)
    H = cfg.hidden
    ones = np.ones(H, dtype=np.float32)
    return {
        "token_embd": blocks(cfg.vocab, H),
        "output": blocks(cfg.vocab, H),
        "output_norm": ones,
        "layers": [{"attn_norm": ones, "qkv": blocks(cfg.qkv_rows, H), "o": blocks(H, cfg.heads * cfg.head_dim),
                    "ffn_norm": ones, "gate_up": blocks(2 * cfg.inter, H), "down": blocks(H, cfg.inter)}
                   for _ in range(cfg.layers)],
    }
