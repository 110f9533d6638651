"""CPU checks of the MusicCoCa style-path oracle (oracle/musiccoca_oracle.cpp)
against an independent torch formulation of the same reference code
(musiccoca.cpp: MusicCoCaEncoder::embed_text; rvq.cpp: rvq_quantization;
style_model.cpp: StyleModel::style_tokens_lm). Random-init text tower with
the reference's key layout, a reduced vocabulary (the gather is the only
place the vocabulary size enters). No GPU needed."""
from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")
F = torch.nn.functional

D, H, DH, FF, LAYERS, POOL_DH, VOCAB, LEVELS = 768, 12, 64, 3072, 12, 256, 1000, 12


def _prompt(rng, n):
    # StyleModel::tokenize_text_ids (style_model.cpp): BOS = 1, then the
    # pieces, zeros after; padding 1.0 on every position after them
    ids = np.zeros((1, 128), np.int32)
    pad = np.ones((1, 128), np.float32)
    ids[0, 0] = 1
    ids[0, 1:n + 1] = rng.integers(2, VOCAB, n)
    pad[0, :n + 1] = 0
    return ids, pad


def _torch_embed_text(w, ids, pad):
    t = {k: torch.from_numpy(v) for k, v in w.items()}

    def mha(p, q_in, kv_in, heads, dh, cap, mask, per_dim):
        B, Sq, _ = q_in.shape
        Sk = kv_in.shape[1]
        q = F.linear(q_in, t[p + ".q_proj.weight"], t[p + ".q_proj.bias"]).view(B, Sq, heads, dh).transpose(1, 2)
        k = F.linear(kv_in, t[p + ".k_proj.weight"], t[p + ".k_proj.bias"]).view(B, Sk, heads, dh).transpose(1, 2)
        v = F.linear(kv_in, t[p + ".v_proj.weight"], t[p + ".v_proj.bias"]).view(B, Sk, heads, dh).transpose(1, 2)
        if per_dim:
            q = q * (F.softplus(t[p + "._per_dim_scale"]) / np.log(2.0))
        a = (q @ k.transpose(-1, -2)) * (1.0 / np.sqrt(dh))
        if cap:
            a = cap * torch.tanh(a / cap)
        if mask is not None:
            a = a + mask
        out = (a.softmax(-1) @ v).transpose(1, 2).reshape(B, Sq, heads * dh)
        return F.linear(out, t[p + ".o_proj.weight"], t[p + ".o_proj.bias"])

    def ln(p, x):
        return F.layer_norm(x, (D,), t[p + ".weight"], t[p + ".bias"], eps=1e-5)

    x = t["token_embedding.weight"][torch.from_numpy(ids).long()] * np.sqrt(D)
    mask = (torch.from_numpy(pad) * -1e9)[:, None, None, :]
    for i in range(LAYERS):
        p = f"text_layers.{i}"
        x = x + mha(p + ".attn", ln(p + ".attn_ln", x), ln(p + ".attn_ln", x), H, DH, 50.0, mask, False)
        h = F.gelu(F.linear(ln(p + ".ffn_ln", x), t[p + ".ffn_w1.weight"], t[p + ".ffn_w1.bias"]))
        x = x + F.linear(h, t[p + ".ffn_w2.weight"], t[p + ".ffn_w2.bias"])
    x = ln("text_exit_ln", x)
    kv = ln("text_pooler.ln", x)
    q = t["text_pooler.query"].expand(x.shape[0], 1, D)
    return mha("text_pooler.attn", q, kv, H, POOL_DH, 0.0, None, True)[:, 0].numpy()


def _rvq(emb, cbs, levels):
    # rvq_quantization (rvq.cpp:24-66) in numpy
    r = emb.astype(np.float32).copy()
    out = []
    for k in range(levels):
        cb = cbs[k]
        d = (r * r).sum(-1, keepdims=True) - 2 * r @ cb.T + (cb * cb).sum(-1)
        tk = d.argmin(-1)
        out.append(tk)
        r = r - cb[tk]
    return np.stack(out, -1).astype(np.int32)


@pytest.mark.parametrize("n_pieces", [3, 40])
def test_embed_text_matches_torch(oracle, style_bundle, n_pieces):
    enc, cb, w = style_bundle
    ids, pad = _prompt(np.random.default_rng(n_pieces), n_pieces)
    o = oracle.StyleOracle(enc, cb)
    got = o.embed_text(ids, pad)
    with torch.no_grad():
        want = _torch_embed_text(w, ids, pad)
    assert got.shape == want.shape == (1, D)
    assert np.isfinite(got).all() and np.abs(want).max() > 1e-2
    assert np.abs(got - want).max() <= 1e-4 * np.abs(want).max(), np.abs(got - want).max()


def test_style_tokens(oracle, mrtdf, style_bundle):
    from safetensors.numpy import load_file

    enc, cb, _ = style_bundle
    o = oracle.StyleOracle(enc, cb)
    ids, pad = _prompt(np.random.default_rng(5), 12)
    emb = o.embed_text(ids, pad)
    tokens = o.quantize(emb, LEVELS)
    np.testing.assert_array_equal(tokens, _rvq(emb, load_file(cb)["codebooks"], LEVELS))
    # StyleModel::style_tokens_lm: the first 6 levels as LLM ids at the style
    # offset 2 + 16 * 1024 + 1024 (system.h:80-82)
    llm = mrtdf.rvq_to_llm(tokens[:, :6], 1024, 17410)
    assert np.all((llm >= 17410 + np.arange(6) * 1024) & (llm < 17410 + (np.arange(6) + 1) * 1024))
    with pytest.raises(RuntimeError):
        o.quantize(emb, LEVELS + 1)


def test_random_bundle_writer_loads_in_the_oracle(oracle, mrtdf, tmp_path, style_bundle):
    """mrtmc.write_random_safetensors writes every key the text tower reads
    with the reference's shapes (same key set as the test bundle)."""
    import mrtmc
    from safetensors.numpy import load_file

    enc, cb = str(tmp_path / "e.safetensors"), str(tmp_path / "c.safetensors")
    mrtmc.write_random_safetensors(enc, cb, seed=1, vocab=500, levels=3)
    got = load_file(enc)
    _, _, want = style_bundle
    assert sorted(got) == sorted(want)
    assert all(got[k].shape == want[k].shape for k in want if k != "token_embedding.weight")
    assert got["token_embedding.weight"].shape == (500, D)
    o = oracle.StyleOracle(enc, cb)
    ids, pad = _prompt(np.random.default_rng(2), 7)
    ids[ids >= 500] = 3
    emb = o.embed_text(ids, pad)
    assert np.isfinite(emb).all()
    assert o.quantize(emb, 3).shape == (1, 3)
    o.close()
