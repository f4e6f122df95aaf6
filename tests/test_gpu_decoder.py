"""Parity of the decode-step kernels of the synthetic MoE decoder (BASELINE
configs[4]) and of a reduced decoder run through frb200.decoder, against fp64
restatements (oracle/).

Tolerances (written here):
  * RMSNorm: max rel err 1e-5;
  * RoPE: q within (2e-5 + 1.5e-7 pos) of max|q| (the angle is formed in f32,
    as ggml and the reference form it, so its rounding grows with pos); the
    appended K rows within one f16 step (2^-10 relative) plus that allowance,
    V rows equal to f16 of the input;
  * decode attention: f16 query and f16 probabilities on the tensor cores
    against fp64 softmax attention over the same f16 K / V: normwise 2e-3,
    max |d| <= 5e-3 * max|ref|;
  * embedding rows bit-exact; arg-max exact (ties to the lowest index);
  * reduced decoder: every stage of a step checked against the oracle fed the
    device's own inputs to that stage (as the reference's FRT_B_HREF mode
    does), matvecs with the dense tolerance (max rel err 1e-3 against
    max(|ref|, 1% rms)), and the whole step replayed from a CUDA graph equal
    to the eager step bit for bit.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _t(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def test_rmsnorm(fr, O, dev):
    import torch
    T, H = 5, 2048
    x = fr.synth_normal(11, T * H).reshape(T, H) * 3.0
    w = fr.synth_normal(12, H)
    y = torch.empty((T, H), dtype=torch.float32, device=dev)
    xd, wd = _t(x, dev), _t(w, dev)             # held: a freed temporary's memory could be reused
    fr.call("fr_rmsnorm_f32", fr._ptr(xd), fr._ptr(wd), fr._ptr(y), T, H, C.c_float(1e-6), fr._stream())
    torch.cuda.synchronize()
    ref = O.rmsnorm(x, w, 1e-6)
    assert np.max(np.abs(y.cpu().numpy() - ref) / (np.abs(ref) + 1e-3)) <= 1e-5


@pytest.mark.parametrize("pos", [0, 1, 37, 1023, 2047])
def test_rope_kv_append(fr, O, dev, pos):
    import torch
    T, nh, nkv, d, ctx = 3, 32, 4, 128, 2048
    qkv = fr.synth_normal(20 + pos, T * (nh + 2 * nkv) * d).reshape(T, (nh + 2 * nkv) * d)
    kc = torch.zeros((T, nkv, ctx, d), dtype=torch.float16, device=dev)
    vc = torch.zeros_like(kc)
    q_r = torch.empty((T, nh, d), dtype=torch.float32, device=dev)
    p = torch.tensor([pos], dtype=torch.int32, device=dev)
    qkvd = _t(qkv, dev)
    fr.call("fr_rope_kv_f16", fr._ptr(qkvd), fr._ptr(p), fr._ptr(q_r), fr._ptr(kc), fr._ptr(vc), T, nh, nkv,
            d, ctx, C.c_float(1e6), fr._stream())
    torch.cuda.synchronize()
    q = qkv[:, : nh * d].reshape(T, nh, d)
    k = qkv[:, nh * d:(nh + nkv) * d].reshape(T, nkv, d)
    v = qkv[:, (nh + nkv) * d:].reshape(T, nkv, d)
    qref = O.rope_neox(q, pos) / np.sqrt(d)
    # the angle pos * theta_scale^i is formed in f32 (as ggml and the
    # reference do): its rounding grows with pos
    tol = (2e-5 + 1.5e-7 * pos) * np.abs(qref).max()
    assert np.max(np.abs(q_r.cpu().numpy() - qref)) <= tol
    kref = O.rope_neox(k, pos)
    kgot = kc[:, :, pos].float().cpu().numpy()
    # f16 rounding of each value plus the same f32-angle allowance as q
    assert np.all(np.abs(kgot - kref) <= np.abs(kref) * 2.0 ** -10 + (2e-5 + 1.5e-7 * pos) * np.abs(kref).max())
    np.testing.assert_array_equal(vc[:, :, pos].cpu().numpy(), v.astype(np.float16))
    # nothing else of the cache was touched
    others = torch.cat([kc[:, :, :pos], kc[:, :, pos + 1:]], 2)
    assert int(torch.count_nonzero(others)) == 0
    assert fr.device_status() == 0


# (T, n_keys): the host splits a sequence's key chunks over 2 * SMs / (T * nkv)
# CTAs (at most ctx / 128), so T = 2 has one chunk per CTA and a split merge,
# T = 24 walks up to 6 chunks per CTA (online softmax) before the merge, and
# T = 64 walks all of them in one CTA with no merge
ATTN_CASES = [(2, n) for n in (1, 2, 127, 128, 129, 300, 1024, 2048)] + \
             [(24, 1), (24, 385), (24, 2048), (64, 1), (64, 129), (64, 1100), (64, 2048)]


@pytest.mark.parametrize("T,n_keys", ATTN_CASES)
def test_attention_decode(fr, O, dev, T, n_keys):
    import torch
    nh, nkv, d, ctx = 32, 4, 128, 2048
    rng = np.random.default_rng(n_keys + 7919 * T)
    q = (rng.standard_normal((T, nh, d)) / np.sqrt(d)).astype(np.float32)
    k = rng.standard_normal((T, nkv, ctx, d)).astype(np.float16)
    v = rng.standard_normal((T, nkv, ctx, d)).astype(np.float16)
    k[:, :, n_keys:] = 0        # the cache beyond the step's keys is zero-initialised
    v[:, :, n_keys:] = 0
    out = torch.empty((T, nh * d), dtype=torch.float32, device=dev)
    p = torch.tensor([n_keys - 1], dtype=torch.int32, device=dev)
    qd, kd, vd = _t(q, dev), _t(k, dev), _t(v, dev)
    for _ in range(2):          # twice: the split counters must be back at zero
        fr.call("fr_attn_decode_f16", fr._ptr(qd), fr._ptr(kd), fr._ptr(vd), fr._ptr(p), fr._ptr(out), T, nh, nkv, d,
                ctx, fr._stream())
        torch.cuda.synchronize()
        got = out.cpu().numpy().reshape(T, nh, d)
        for t in range(T):
            ref = O.attention_decode(q[t], k[t, :, :n_keys], v[t, :, :n_keys])
            nerr = np.linalg.norm(got[t] - ref) / np.linalg.norm(ref)
            assert nerr <= 2e-3, f"t={t}: normwise {nerr:.2e}"
            assert np.max(np.abs(got[t] - ref)) <= 5e-3 * np.abs(ref).max()
    assert fr.device_status() == 0


def test_embed_rows_and_argmax(fr, O, dev):
    import torch
    V, H, T, P = 1000, 512, 3, 4
    table = fr.synth_nvfp4(31, V, H)
    prompt = np.array([[5, 999, 0, 17], [1, 2, 3, 4], [998, 7, 7, 500]], np.int32)
    gen = torch.tensor([42, 0, 999], dtype=torch.int32, device=dev)
    x = torch.empty((T, H), dtype=torch.float32, device=dev)
    tab = _t(table, dev)
    pr = _t(prompt, dev)
    for pos in (0, 3, 4):       # prompt, last prompt token, then the generated tokens
        p = torch.tensor([pos], dtype=torch.int32, device=dev)
        fr.call("fr_embed_nvfp4", fr._ptr(tab), V, H, fr._ptr(pr), P, P, fr._ptr(gen), fr._ptr(p), fr._ptr(x), T,
                fr._stream())
        torch.cuda.synchronize()
        toks = prompt[:, pos] if pos < P else gen.cpu().numpy()
        np.testing.assert_array_equal(x.cpu().numpy(), O.nvfp4_rows(table, toks).reshape(T, H))
    logits = fr.synth_normal(32, T * V).reshape(T, V)
    logits[1, 10] = logits[1, 700] = logits[1].max() + 1.0      # a tie: the lower index wins
    tok = torch.empty(T, dtype=torch.int32, device=dev)
    ld = _t(logits, dev)
    fr.call("fr_argmax_f32", fr._ptr(ld), T, V, fr._ptr(tok), fr._stream())
    torch.cuda.synchronize()
    np.testing.assert_array_equal(tok.cpu().numpy(), np.argmax(logits, 1))
    assert int(tok[1]) == 10
    assert fr.device_status() == 0


def _matvec_check(O, mine, w, xin, N, K, what):
    ref = O.gemv_q8_1(w, O.quantize_q8_1(np.ascontiguousarray(xin, np.float32)), N, K)
    err = O.rel_err(mine, ref)
    assert err <= 1e-3, f"{what}: max rel err {err:.3e}"


@pytest.mark.parametrize("dense,experts", [("ggml", "ggml"), ("tiled", "tiled")])
def test_reduced_decoder_stagewise(fr, O, dev, dense, experts):
    """A 2-layer decoder (hidden 512, 8 query / 1 KV heads of 128, 32 experts
    top-4 of FFN 256, vocab 1024, ctx 256): a 3-token prompt and 2 decode
    steps; the last step re-run stage by stage with the checks in the module
    docstring; graph replay equal to eager."""
    import torch
    from frb200.decoder import Config, MoeDecoder
    cfg = Config(n_layers=2, hidden=512, n_head=8, n_kv=1, head_dim=128, n_expert=32, n_used=4, n_ff=256,
                 vocab=1024, ctx=256)
    T = 2
    dec = MoeDecoder(cfg, T, seed=0x5EED6000, dense=dense, experts=experts)
    prompt = torch.tensor([[3, 1000, 77], [5, 5, 1023]], dtype=torch.int32, device=dev)
    dec.set_prompt(prompt)
    for _ in range(4):
        dec.step()
    torch.cuda.synchronize()
    assert int(dec.pos) == 4 and fr.device_status() == 0
    toks_eager = dec.tok.clone()
    x_eager = dec.x[0].clone()

    # the same 4 steps replayed from one captured step
    dec.set_prompt(prompt)
    dec.kc.zero_()
    dec.vc.zero_()
    s = torch.cuda.Stream(dev)
    with torch.cuda.stream(s):
        dec.step(stream=s)          # warm-up (workspaces)
    s.synchronize()
    dec.set_prompt(prompt)
    dec.kc.zero_()
    dec.vc.zero_()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        dec.step(stream=s)
    dec.pos.zero_()
    dec.kc.zero_()
    dec.vc.zero_()
    torch.cuda.synchronize()
    for _ in range(4):
        g.replay()
    torch.cuda.synchronize()
    assert torch.equal(dec.tok, toks_eager)
    assert torch.equal(dec.x[0], x_eager)
    del g

    # step 5 (pos 4, decoding) stage by stage, layer 0, on the host oracle
    H, d = cfg.hidden, cfg.head_dim
    lay = dec.layers[0]
    x0 = torch.empty((T, H), dtype=torch.float32, device=dev)
    fr.call("fr_embed_nvfp4", fr._ptr(dec.embed), cfg.vocab, H, None, 0, 0, fr._ptr(dec.tok), fr._ptr(dec.pos),
            fr._ptr(x0), T, fr._stream())
    xn = torch.empty_like(x0)
    fr.call("fr_rmsnorm_f32", fr._ptr(x0), fr._ptr(dec.norm_w), fr._ptr(xn), T, H, C.c_float(cfg.eps), fr._stream())
    qkv = torch.empty((T, cfg.qkv_width), dtype=torch.float32, device=dev)
    dec._matvec(lay["wqkv"], xn, cfg.qkv_width, H, qkv)
    q_r = torch.empty((T, cfg.n_head, d), dtype=torch.float32, device=dev)
    fr.call("fr_rope_kv_f16", fr._ptr(qkv), fr._ptr(dec.pos), fr._ptr(q_r), fr._ptr(dec.kc[0]), fr._ptr(dec.vc[0]), T,
            cfg.n_head, cfg.n_kv, d, cfg.ctx, C.c_float(cfg.rope_base), fr._stream())
    att = torch.empty((T, cfg.n_head * d), dtype=torch.float32, device=dev)
    fr.call("fr_attn_decode_f16", fr._ptr(q_r), fr._ptr(dec.kc[0]), fr._ptr(dec.vc[0]), fr._ptr(dec.pos),
            fr._ptr(att), T, cfg.n_head, cfg.n_kv, d, cfg.ctx, fr._stream())
    x2 = torch.empty_like(x0)
    dec._matvec(lay["wo"], att, H, cfg.n_head * d, x2, resid=x0)
    torch.cuda.synchronize()
    hx0, hxn, hqkv = x0.cpu().numpy(), xn.cpu().numpy(), qkv.cpu().numpy()
    assert np.max(np.abs(hxn - O.rmsnorm(hx0, None, cfg.eps)) / (np.abs(hxn) + 1e-3)) <= 1e-5
    if dense == "ggml":
        _matvec_check(O, hqkv, lay["wqkv"].cpu().numpy(), hxn, cfg.qkv_width, H, "qkv")
    pos = int(dec.pos)
    kc, vc = dec.kc[0].float().cpu().numpy(), dec.vc[0].float().cpu().numpy()
    for t in range(T):
        q = O.rope_neox(hqkv[t, : cfg.n_head * d].reshape(cfg.n_head, d), pos) / np.sqrt(d)
        assert np.max(np.abs(q_r.cpu().numpy()[t] - q)) <= (2e-5 + 1.5e-7 * pos) * np.abs(q).max()
        ref = O.attention_decode(q_r.cpu().numpy()[t], kc[t, :, : pos + 1], vc[t, :, : pos + 1])
        got = att.cpu().numpy()[t].reshape(cfg.n_head, d)
        assert np.linalg.norm(got - ref) / np.linalg.norm(ref) <= 2e-3
    if dense == "ggml":
        ref = O.gemv_q8_1(lay["wo"].cpu().numpy(), O.quantize_q8_1(att.cpu().numpy()), H, cfg.n_head * d) + hx0
        assert O.rel_err(x2.cpu().numpy(), ref) <= 1e-3
    assert fr.device_status() == 0
