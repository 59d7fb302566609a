"""CPU reference of the Q8_0 decoder: one batch-1 decode step, and the prompt pass.

TEST INFRASTRUCTURE ONLY (see q8_0_oracle.c): the checker for
talechime_b200/decoder.py.  Restates crates/voxcpm/src/transformer.rs:107-155 (layer
loop), :40-41 (rms_norm, candle_nn::ops::rms_norm: sequential f32 sum of squares,
m = sqrt(sum/n + eps), y = x / m * w), :44-65 and :159-170 (RoPE tables and rotation
x*[cos,cos] + [second,first]*[-sin,sin]), attention.rs:28-98 (scores = q k^T times the f32
rounding of 1/sqrt(d), softmax over the last dim in f32, times v; kv head = q head /
(Hq/Hkv)), with every Q8_0 linear computed by the C oracle (candle's CPU QMatMul) and
SwiGLU by the oracle's silu.  f32 throughout; the GPU path is checked against it within
tolerance.
"""
from __future__ import annotations

import numpy as np

import oracle


def _rms_norm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    x = x.astype(np.float32)
    sum2 = np.add.accumulate((x * x).astype(np.float32), dtype=np.float32)[-1]
    m = np.float32(np.sqrt(np.float32(sum2 / np.float32(x.size) + np.float32(eps))))
    return ((x / m).astype(np.float32) * w.astype(np.float32)).astype(np.float32)


def _dequant_row(blocks: np.ndarray, row: int, k: int) -> np.ndarray:
    b = np.ascontiguousarray(blocks.reshape(-1, k // 32, 34)[row])
    return oracle.dequantize(b.reshape(1, -1), k).reshape(-1)


class DecoderRef:
    """Holds the f32 KV cache of the reference decode."""

    def __init__(self, cfg, weights: dict, cos: np.ndarray, sin: np.ndarray):
        self.cfg, self.w, self.cos, self.sin = cfg, weights, cos, sin
        self.k = [np.zeros((cfg.kv_heads, cfg.max_t, cfg.head_dim), np.float32) for _ in range(cfg.layers)]
        self.v = [np.zeros((cfg.kv_heads, cfg.max_t, cfg.head_dim), np.float32) for _ in range(cfg.layers)]

    def _rope(self, x: np.ndarray, pos: int) -> np.ndarray:
        half = self.cfg.head_dim // 2
        c = np.concatenate([self.cos[pos], self.cos[pos]]).astype(np.float32)
        s = np.concatenate([-self.sin[pos], self.sin[pos]]).astype(np.float32)
        swapped = np.concatenate([x[..., half:], x[..., :half]], axis=-1)
        return ((x * c).astype(np.float32) + (swapped * s).astype(np.float32)).astype(np.float32)

    def step(self, token: int, pos: int) -> np.ndarray:
        """Logits f32 [vocab] for `token` at `pos` (appends to the cache)."""
        cfg, w = self.cfg, self.w
        H, D, Hq, Hk = cfg.hidden, cfg.head_dim, cfg.heads, cfg.kv_heads
        scale = np.float32(1.0 / np.sqrt(float(D)))
        x = _dequant_row(np.asarray(w["token_embd"]), token, H)
        for li in range(cfg.layers):
            lw = w["layers"][li]
            h = _rms_norm(x, np.asarray(lw["attn_norm"]), cfg.eps)
            qkv = oracle.matmul(h[None, :], np.asarray(lw["qkv"]), cfg.qkv_rows)[0]
            q = self._rope(qkv[:Hq * D].reshape(Hq, D), pos)
            k = self._rope(qkv[Hq * D:(Hq + Hk) * D].reshape(Hk, D), pos)
            v = qkv[(Hq + Hk) * D:].reshape(Hk, D)
            self.k[li][:, pos] = k
            self.v[li][:, pos] = v
            out = np.empty((Hq, D), np.float32)
            for hh in range(Hq):
                kh = hh // (Hq // Hk)
                sc = (self.k[li][kh, :pos + 1] @ q[hh]).astype(np.float32) * scale
                e = np.exp((sc - sc.max()).astype(np.float32)).astype(np.float32)
                p = (e / e.sum(dtype=np.float32)).astype(np.float32)
                out[hh] = (p @ self.v[li][kh, :pos + 1]).astype(np.float32)
            o = oracle.matmul(out.reshape(1, -1), np.asarray(lw["o"]), H)[0]
            x = (x + o).astype(np.float32)
            h = _rms_norm(x, np.asarray(lw["ffn_norm"]), cfg.eps)
            gu = oracle.matmul(h[None, :], np.asarray(lw["gate_up"]), 2 * cfg.inter)
            d = oracle.matmul(oracle.swiglu(gu), np.asarray(lw["down"]), H)[0]
            x = (x + d).astype(np.float32)
        h = _rms_norm(x, np.asarray(w["output_norm"]), cfg.eps)
        return oracle.matmul(h[None, :], np.asarray(w["output"]), cfg.vocab)[0]

    def prefill(self, tokens, pos0: int) -> np.ndarray:
        """Logits f32 [vocab] of the last of `tokens`, run as ONE forward of T = len(tokens)
        rows at positions pos0 .. pos0 + T - 1 (the prompt pass of crates/voxcpm/src/
        model.rs:492-495 through transformer.rs:107-155 with offset = pos0): every linear
        takes all T rows at once (candle's QMatMul quantizes and dots each row on its
        own), RoPE rotates row i at position pos0 + i, the cache grows by T rows, and row
        i attends to cache rows [0, pos0 + i] (the causal mask of attention.rs:84-95
        excludes key j when j > offset + i); the caller's next token comes from the last
        row (the reference's norm -> head on x[:, t - 1])."""
        cfg, w = self.cfg, self.w
        H, D, Hq, Hk = cfg.hidden, cfg.head_dim, cfg.heads, cfg.kv_heads
        T = len(tokens)
        if pos0 < 0 or pos0 + T > cfg.max_t:
            raise ValueError("Transformer context limit exceeded")
        scale = np.float32(1.0 / np.sqrt(float(D)))
        x = np.stack([_dequant_row(np.asarray(w["token_embd"]), int(t), H) for t in tokens]).astype(np.float32)
        for li in range(cfg.layers):
            lw = w["layers"][li]
            h = np.stack([_rms_norm(r, np.asarray(lw["attn_norm"]), cfg.eps) for r in x])
            qkv = oracle.matmul(h, np.asarray(lw["qkv"]), cfg.qkv_rows)
            q = np.empty((T, Hq, D), np.float32)
            for i in range(T):
                q[i] = self._rope(qkv[i, :Hq * D].reshape(Hq, D), pos0 + i)
                self.k[li][:, pos0 + i] = self._rope(qkv[i, Hq * D:(Hq + Hk) * D].reshape(Hk, D), pos0 + i)
                self.v[li][:, pos0 + i] = qkv[i, (Hq + Hk) * D:].reshape(Hk, D)
            att = np.empty((T, Hq, D), np.float32)
            for hh in range(Hq):
                kh = hh // (Hq // Hk)
                for i in range(T):
                    n = pos0 + i + 1  # visible keys
                    sc = (self.k[li][kh, :n] @ q[i, hh]).astype(np.float32) * scale
                    e = np.exp((sc - sc.max()).astype(np.float32)).astype(np.float32)
                    p = (e / e.sum(dtype=np.float32)).astype(np.float32)
                    att[i, hh] = (p @ self.v[li][kh, :n]).astype(np.float32)
            o = oracle.matmul(att.reshape(T, Hq * D), np.asarray(lw["o"]), H)
            x = (x + o).astype(np.float32)
            h = np.stack([_rms_norm(r, np.asarray(lw["ffn_norm"]), cfg.eps) for r in x])
            gu = oracle.matmul(h, np.asarray(lw["gate_up"]), 2 * cfg.inter)
            d = oracle.matmul(oracle.swiglu(gu), np.asarray(lw["down"]), H)
            x = (x + d).astype(np.float32)
        h = _rms_norm(x[T - 1], np.asarray(w["output_norm"]), cfg.eps)
        return oracle.matmul(h[None, :], np.asarray(w["output"]), cfg.vocab)[0]
