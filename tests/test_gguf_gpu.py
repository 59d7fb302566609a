"""GGUF -> device weights: q8lin_gguf_weight_create and Q8Decoder.from_gguf."""
import numpy as np
import pytest
import torch

from talechime_b200 import QMatMul, synth
from talechime_b200._lib import Q8LinError
from talechime_b200.decoder import DecoderConfig, Q8Decoder, rope_tables
from talechime_b200.gguf import GGUFFile
from tests import gguf_writer as gw

pytestmark = pytest.mark.gpu


def test_linear_from_gguf_is_the_uploaded_tensor(tmp_path, cuda_device):
    rng = np.random.default_rng(60)
    n, k = 300, 2048
    blocks = synth.q8_0_blocks(rng, n, k)
    path = gw.Writer(alignment=64).q8_0("blk.3.ffn_down.weight", blocks, k).write(tmp_path / "w.gguf")
    with GGUFFile(path) as g:
        a = g.linear("blk.3.ffn_down", device=cuda_device)
        with pytest.raises(Q8LinError):
            g.linear("blk.3.ffn_up", device=cuda_device)
    b = QMatMul.from_gguf_blocks(blocks, n, k, device=cuda_device)
    assert a.shape() == (n, k)
    assert torch.equal(a.to_gguf_blocks().cpu(), b.to_gguf_blocks().cpu())
    x = torch.from_numpy(rng.standard_normal((3, k)).astype(np.float32)).to(cuda_device)
    assert torch.equal(a.forward(x), b.forward(x))


def _write_decoder(path, cfg, w, factors):
    """A GGUF file with the reference's BaseLM tensor names (q/k/v and gate/up unfused)."""
    wr = gw.Writer()
    wr.add("general.architecture", gw.STRING, "minicpm4")
    for key, val in [("embedding_length", cfg.hidden), ("block_count", cfg.layers),
                     ("feed_forward_length", cfg.inter), ("vocab_size", cfg.vocab),
                     ("attention.head_count", cfg.heads), ("attention.head_count_kv", cfg.kv_heads),
                     ("attention.key_length", cfg.head_dim), ("attention.value_length", cfg.head_dim)]:
        wr.add(f"minicpm4.{key}", gw.U32, val)
    H, D = cfg.hidden, cfg.head_dim
    wr.q8_0("token_embd.weight", w["token_embd"], H)
    wr.f32("rope_factors_short.weight", factors)
    for i, lw in enumerate(w["layers"]):
        qkv = lw["qkv"].reshape(cfg.qkv_rows, -1)
        nq, nk = cfg.heads * D, cfg.kv_heads * D
        wr.f32(f"blk.{i}.attn_norm.weight", lw["attn_norm"])
        wr.q8_0(f"blk.{i}.attn_q.weight", qkv[:nq], H)
        wr.q8_0(f"blk.{i}.attn_k.weight", qkv[nq:nq + nk], H)
        wr.q8_0(f"blk.{i}.attn_v.weight", qkv[nq + nk:], H)
        wr.q8_0(f"blk.{i}.attn_output.weight", lw["o"], cfg.heads * D)
        wr.f32(f"blk.{i}.ffn_norm.weight", lw["ffn_norm"])
        gu = lw["gate_up"].reshape(2 * cfg.inter, -1)
        wr.q8_0(f"blk.{i}.ffn_gate.weight", gu[:cfg.inter], H)
        wr.q8_0(f"blk.{i}.ffn_up.weight", gu[cfg.inter:], H)
        wr.q8_0(f"blk.{i}.ffn_down.weight", lw["down"], cfg.inter)
    wr.f32("output_norm.weight", w["output_norm"])
    wr.q8_0("output.weight", w["output"], H)
    return wr.write(path)


def test_decoder_from_gguf_matches_reference(tmp_path, oracle_lib, cuda_device):
    from oracle.decoder_ref import DecoderRef
    from tests.test_decoder_gpu import LOGITS_REL_L2, _rel, _tiny

    cfg, w = _tiny(4, 2, 70)
    cfg = DecoderConfig(**{**cfg.__dict__, "max_t": 16})
    factors = np.random.default_rng(71).uniform(1.0, 4.0, cfg.head_dim // 2).astype(np.float32)
    path = _write_decoder(tmp_path / "base.gguf", cfg, w, factors)
    dec = Q8Decoder.from_gguf(path, device=cuda_device, max_t=16,
                              expect={"block_count": cfg.layers, "attention.head_count_kv": 2})
    assert dec.cfg == cfg
    with pytest.raises(Q8LinError, match="unsupported GGUF minicpm4.block_count=2; expected 28"):
        Q8Decoder.from_gguf(path, device=cuda_device, expect={"block_count": 28})
    cos, sin = rope_tables(cfg, factors)
    ref = DecoderRef(cfg, w, cos, sin)
    dec.reset(11)
    tok = 11
    for pos in range(6):
        dec.step()
        lr = ref.step(tok, pos)
        assert _rel(dec.logits.cpu().numpy(), lr) <= LOGITS_REL_L2, pos
        tok = int(dec.token.item())
        assert tok == int(np.argmax(lr))
