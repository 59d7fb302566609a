"""Batched prefill of the decoder (csrc/prefill.cu, Q8Decoder.prefill) against the CPU
reference's prompt pass (oracle/decoder_ref.py: crates/voxcpm/src/model.rs:492-495 through
transformer.rs:107-155 with the causal mask of attention.rs:84-95)."""
import ctypes

import numpy as np
import pytest
import torch

from talechime_b200 import _lib
from talechime_b200.decoder import DecoderConfig, Q8Decoder, rope_tables, synthetic_weights

pytestmark = pytest.mark.gpu

# whole-model logits: see tests/test_decoder_gpu.py (one re-quantization per linear)
LOGITS_REL_L2 = 2e-3
FLIP_REL_L2 = 3e-2


def _s():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _rel(a, b):
    return float(np.linalg.norm(np.asarray(a, np.float64) - b) / np.linalg.norm(b))


def _rope_np(x, pos, cos, sin):
    """x [.., D] rotated at `pos` with candle's rounding (each product rounded, then added)."""
    half = x.shape[-1] // 2
    c = np.concatenate([cos[pos], cos[pos]]).astype(np.float32)
    s = np.concatenate([-sin[pos], sin[pos]]).astype(np.float32)
    sw = np.concatenate([x[..., half:], x[..., :half]], axis=-1)
    return ((x * c).astype(np.float32) + (sw * s).astype(np.float32)).astype(np.float32)


@pytest.mark.parametrize("D", [128, 100], ids=["float4_kernel", "scalar_kernel"])
def test_rope_kv_rows_is_the_reference_rotation(cuda_device, D):
    """Every row rotated at its own position (bit-exact), k and v appended at rows
    pos0 .. pos0 + T - 1 of their sequence's cache, every other cache row untouched
    (D = 128 takes the float4 kernel, D = 100 the scalar one)."""
    B, T, pos0, hq, hkv, max_t = 2, 5, 3, 4, 2, 16
    cfg = DecoderConfig(hidden=256, layers=1, heads=hq, kv_heads=hkv, head_dim=D, inter=256, vocab=8, max_t=max_t)
    cos, sin = rope_tables(cfg)
    rng = np.random.default_rng(3)
    qkv = rng.standard_normal((B * T, (hq + 2 * hkv) * D), dtype=np.float32)
    dev = cuda_device
    kc = torch.full((B, hkv, max_t, D), 7.0, device=dev)
    vc = torch.full((B, hkv, max_t, D), -7.0, device=dev)
    q_out = torch.empty((B * T, hq, D), device=dev)
    L = _lib.lib()
    # device copies held in names: a temporary freed inside the argument list would hand
    # its memory to the next argument's allocation before the kernel runs
    qkv_d, cos_d, sin_d = (torch.from_numpy(a).to(dev) for a in (qkv, cos, sin))
    _lib.check(L.q8lin_rope_kv_rows(_p(qkv_d), B, T, pos0, _p(cos_d), _p(sin_d), _p(kc), _p(vc), hq, hkv, D, max_t,
                                    _p(q_out), _s()))
    torch.cuda.synchronize()
    kc, vc, q_out = kc.cpu().numpy(), vc.cpu().numpy(), q_out.cpu().numpy()
    for b in range(B):
        for t in range(T):
            r, pos = b * T + t, pos0 + t
            row = qkv[r].reshape(hq + 2 * hkv, D)
            assert np.array_equal(q_out[r], _rope_np(row[:hq], pos, cos, sin))
            assert np.array_equal(kc[b, :, pos], _rope_np(row[hq:hq + hkv], pos, cos, sin))
            assert np.array_equal(vc[b, :, pos], row[hq + hkv:])
    untouched = np.ones(max_t, bool)
    untouched[pos0:pos0 + T] = False
    assert np.all(kc[:, :, untouched] == 7.0) and np.all(vc[:, :, untouched] == -7.0)


@pytest.mark.parametrize("m,n", [(3, 2048), (5, 6144), (2, 100)], ids=["hidden", "inter", "unaligned_width"])
def test_add_rmsnorm_is_add_then_rmsnorm(cuda_device, m, n):
    """x += y; h = x / sqrt(sum(x^2)/n + eps) * w: the sum exact per element (bit-exact x),
    h against float64 within f32 summation-order tolerance (n = 100 takes the add and
    rmsnorm kernels)."""
    rng = np.random.default_rng(m + n)
    x, y = rng.standard_normal((m, n), dtype=np.float32), rng.standard_normal((m, n), dtype=np.float32)
    w = rng.uniform(0.5, 1.5, n).astype(np.float32)
    dev = cuda_device
    xd, yd, wd = (torch.from_numpy(a).to(dev) for a in (x, y, w))
    hd = torch.empty((m, n), device=dev)
    _lib.check(_lib.lib().q8lin_add_rmsnorm(_p(xd), _p(yd), _p(wd), m, n, 1e-5, _p(hd), _s()))
    xs = (x + y).astype(np.float32)
    assert np.array_equal(xd.cpu().numpy(), xs)
    x64 = xs.astype(np.float64)
    ref = x64 / np.sqrt((x64 * x64).sum(1, keepdims=True) / n + 1e-5) * w
    np.testing.assert_allclose(hd.cpu().numpy(), ref, rtol=2e-6, atol=1e-6)


def _attention_np(q, kc, vc, T, pos0, hq, hkv):
    """float64 causal grouped attention: row i of a sequence sees cache rows [0, pos0 + i]."""
    B = kc.shape[0]
    D = q.shape[-1]
    scale = np.float64(np.float32(1.0 / np.sqrt(128.0)))
    out = np.empty(q.shape, np.float64)
    for b in range(B):
        for h in range(hq):
            kh = h // (hq // hkv)
            for i in range(T):
                n = pos0 + i + 1
                sc = kc[b, kh, :n].astype(np.float64) @ q[b * T + i, h].astype(np.float64) * scale
                e = np.exp(sc - sc.max())
                out[b * T + i, h] = (e / e.sum()) @ vc[b, kh, :n].astype(np.float64)
    return out


@pytest.mark.parametrize("B,T,pos0,hq,hkv,max_t", [
    (1, 1, 0, 2, 2, 8),        # one row, one key
    (1, 64, 0, 16, 2, 64),     # one full tile, GQA 8:1, cache exactly full
    (2, 100, 37, 4, 2, 200),   # offset prefill (a chunk after 37 cached rows), partial tiles
    (1, 130, 5, 16, 2, 160),   # three query tiles, the last with 2 rows
    (3, 65, 0, 8, 8, 80),      # no grouping, a 1-row last tile
    (1, 200, 300, 2, 1, 512),  # long history before the new rows
    (6, 200, 10, 16, 16, 256),  # 384 CTAs at 64-row tiles (the cases above take 32-row tiles)
])
def test_attention_prefill_matches_masked_softmax(cuda_device, B, T, pos0, hq, hkv, max_t):
    """Cache rows past pos0 + T hold NaN: the kernel must never let them into a sum."""
    D = 128
    rng = np.random.default_rng(B * 1000 + T + pos0)
    q = rng.standard_normal((B * T, hq, D), dtype=np.float32)
    kc = np.full((B, hkv, max_t, D), np.nan, np.float32)
    vc = np.full((B, hkv, max_t, D), np.nan, np.float32)
    kc[:, :, :pos0 + T] = rng.standard_normal((B, hkv, pos0 + T, D), dtype=np.float32)
    vc[:, :, :pos0 + T] = rng.standard_normal((B, hkv, pos0 + T, D), dtype=np.float32)
    dev = cuda_device
    out = torch.full((B * T, hq, D), np.nan, device=dev)
    q_d, kc_d, vc_d = (torch.from_numpy(a).to(dev) for a in (q, kc, vc))
    _lib.check(_lib.lib().q8lin_attention_prefill(_p(q_d), _p(kc_d), _p(vc_d), B, T, pos0, hq, hkv, D, max_t, _p(out),
                                                  _s()))
    got = out.cpu().numpy()
    ref = _attention_np(q, kc, vc, T, pos0, hq, hkv)
    assert np.isfinite(got).all()
    # f32 dot products of 128 terms and an online softmax against float64
    np.testing.assert_allclose(got, ref, rtol=1e-4, atol=2e-6 * np.abs(ref).max())
    assert _rel(got, ref) <= 1e-5


def _tiny(seed, max_t=24, batch=1):
    cfg = DecoderConfig(hidden=256, layers=2, heads=4, kv_heads=2, inter=512, vocab=1000, max_t=max_t)
    w = synthetic_weights(cfg, seed=seed)
    rng = np.random.default_rng(seed + 1)
    w["output_norm"] = rng.uniform(0.5, 1.5, cfg.hidden).astype(np.float32)
    for lw in w["layers"]:
        lw["attn_norm"] = rng.uniform(0.5, 1.5, cfg.hidden).astype(np.float32)
        lw["ffn_norm"] = rng.uniform(0.5, 1.5, cfg.hidden).astype(np.float32)
    return cfg, w


def test_prefill_matches_reference_prompt_pass(oracle_lib, cuda_device):
    """A 10-token prompt, a 5-token continuation chunk at offset 10 (the reference's cache
    path with offset > 0), then decode steps: logits, next tokens and cache rows against
    the CPU reference."""
    from oracle.decoder_ref import DecoderRef

    cfg, w = _tiny(61)
    dec = Q8Decoder(cfg, w, device=cuda_device)
    ref = DecoderRef(cfg, w, *rope_tables(cfg))
    rng = np.random.default_rng(62)
    pos = 0
    for chunk in (rng.integers(0, cfg.vocab, 10), rng.integers(0, cfg.vocab, 5)):
        nxt = dec.prefill(chunk)
        lr = ref.prefill(chunk, pos)
        pos += len(chunk)
        assert _rel(dec.logits.cpu().numpy(), lr) <= LOGITS_REL_L2
        assert int(nxt.item()) == int(np.argmax(lr)) == int(dec.token.item())
        assert int(dec.pos.item()) == pos
        for li in range(cfg.layers):
            assert _rel(dec.k_cache[li][:, :pos].cpu().numpy(), ref.k[li][:, :pos]) <= LOGITS_REL_L2
            assert _rel(dec.v_cache[li][:, :pos].cpu().numpy(), ref.v[li][:, :pos]) <= LOGITS_REL_L2
    tok = int(dec.token.item())
    for _ in range(4):  # decoding continues from the prefilled state
        dec.step()
        lr = ref.step(tok, pos)
        pos += 1
        assert _rel(dec.logits.cpu().numpy(), lr) <= LOGITS_REL_L2
        tok = int(dec.token.item())
        assert tok == int(np.argmax(lr))


def test_prefill_sequences_of_a_batch_are_independent(oracle_lib, cuda_device):
    """batch = 3: each sequence against the CPU reference's prompt pass of that sequence
    alone, and against a batch-1 GPU prefill of it (the linears then run at M = 3T instead
    of T: another kernel).  At hidden 256 one activation of sequence 1 sits on a Q8_0
    rounding boundary -- 1e-7 relative noise on the reference's own input moves its
    logits by 1.1e-2 -- so whole-model comparisons take the flip bound; layer 0's cache
    rows of the two GPU runs come from bit-identical quantized activations and agree
    tightly."""
    from oracle.decoder_ref import DecoderRef

    cfg, w = _tiny(71)
    T = 9
    toks = np.random.default_rng(72).integers(0, cfg.vocab, (3, T))
    big = Q8Decoder(cfg, w, device=cuda_device, batch=3)
    nxt = big.prefill(toks).cpu().numpy()
    assert int(big.pos.item()) == T
    with pytest.raises(ValueError):
        big.step()
    for b in range(3):
        ref = DecoderRef(cfg, w, *rope_tables(cfg))
        lr = ref.prefill(toks[b], 0)
        lb = big.prefill_logits[b].cpu().numpy()
        assert _rel(lb, lr) <= FLIP_REL_L2, b
        top2 = np.sort(lr)[-2:]
        if top2[1] - top2[0] > 1e-2 * abs(top2[1]):  # a clear winner
            assert nxt[b] == int(np.argmax(lr)), b
        one = Q8Decoder(cfg, w, device=cuda_device)
        one.prefill(toks[b])
        assert _rel(lb, one.logits.cpu().numpy().astype(np.float64)) <= FLIP_REL_L2, b
        for li in range(cfg.layers):
            kb, vb = big.k_cache[li][b, :, :T].cpu().numpy(), big.v_cache[li][b, :, :T].cpu().numpy()
            assert _rel(kb, ref.k[li][:, :T]) <= FLIP_REL_L2 and _rel(vb, ref.v[li][:, :T]) <= FLIP_REL_L2
            k1 = one.k_cache[li][:, :T].cpu().numpy().astype(np.float64)
            assert _rel(kb, k1) <= (1e-5 if li == 0 else FLIP_REL_L2), (b, li)


def test_prefill_launches_replay_from_a_cuda_graph(cuda_device):
    """The launches of a prefill synchronise nothing: after one warm-up call of the same
    size they capture into a CUDA graph, and a replay leaves exactly the state of an eager
    prefill (next token, logits, cache rows, position)."""
    cfg, w = _tiny(101)
    toks = np.random.default_rng(102).integers(0, cfg.vocab, 11)
    eager = Q8Decoder(cfg, w, device=cuda_device)
    n_eager = int(eager.prefill(toks).item())
    dec = Q8Decoder(cfg, w, device=cuda_device)
    dec.prefill(toks)  # warm-up: workspaces and kernel attributes before the capture
    dec.reset()
    tok_d = torch.tensor(toks, dtype=torch.int32, device=cuda_device)
    stream = torch.cuda.Stream(cuda_device)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        dec.logits.zero_()
        for li in range(cfg.layers):
            dec.k_cache[li].zero_()
            dec.v_cache[li].zero_()
        torch.cuda.synchronize()
        with torch.cuda.graph(graph, stream=stream):
            dec._prefill_launches(tok_d, 1, len(toks), 0)
        graph.replay()
        torch.cuda.synchronize()
    assert int(dec.token.item()) == n_eager and int(dec.pos.item()) == len(toks)
    assert torch.equal(dec.logits, eager.logits)
    for li in range(cfg.layers):
        assert torch.equal(dec.k_cache[li][:, :len(toks)], eager.k_cache[li][:, :len(toks)])
        assert torch.equal(dec.v_cache[li][:, :len(toks)], eager.v_cache[li][:, :len(toks)])
    del graph


def test_prefill_context_limit_and_shapes(cuda_device):
    cfg, w = _tiny(81, max_t=12)
    dec = Q8Decoder(cfg, w, device=cuda_device)
    dec.prefill([1, 2, 3, 4, 5, 6, 7, 8])
    with pytest.raises(_lib.Q8LinError) as e:
        dec.prefill([1, 2, 3, 4, 5])  # 8 + 5 > 12
    assert e.value.status == _lib.ERR_SHAPE
    assert int(dec.pos.item()) == 8  # nothing ran
    with pytest.raises(_lib.Q8LinError):
        dec.prefill(np.zeros((2, 2), np.int64))  # batch 1 decoder


def test_prefill_equals_decode_steps_at_full_width(cuda_device):
    """Full widths (hidden 2048, GQA 16:2, MLP 6144): a 128-token prefill (M = 128 linears,
    two query tiles) against 128 decode steps over the same tokens (M = 1 linears, the
    decode attention kernel) -- two independent code paths to the same state."""
    cfg = DecoderConfig(hidden=2048, layers=2, heads=16, kv_heads=2, inter=6144, vocab=4096, max_t=160)
    w = synthetic_weights(cfg, seed=91, device=cuda_device)
    rng = np.random.default_rng(92)
    for lw in w["layers"]:
        lw["attn_norm"] = rng.uniform(0.5, 1.5, cfg.hidden).astype(np.float32)
        lw["ffn_norm"] = rng.uniform(0.5, 1.5, cfg.hidden).astype(np.float32)
    toks = rng.integers(0, cfg.vocab, 128)
    a = Q8Decoder(cfg, w, device=cuda_device)
    b = Q8Decoder(cfg, w, device=cuda_device)
    a.prefill(toks)
    for t in toks:
        b.token.fill_(int(t))
        b.step(mode="fused")
    torch.cuda.synchronize()
    assert int(a.pos.item()) == int(b.pos.item()) == 128
    # layer 0's cache rows depend only on the embedding, one norm and the qkv linear
    for ca, cb in ((a.k_cache[0], b.k_cache[0]), (a.v_cache[0], b.v_cache[0])):
        assert _rel(ca[:, :128].cpu().numpy(), cb[:, :128].double().cpu().numpy()) <= 1e-4
    assert _rel(a.logits.cpu().numpy(), b.logits.cpu().numpy().astype(np.float64)) <= FLIP_REL_L2
    st = ctypes.c_uint32(0)
    _lib.check(_lib.lib().q8lin_fault_status(torch.cuda.current_device(), ctypes.byref(st), 1))
    assert st.value == 0
