"""GGUF reader / writer and the tensor-parallel shard cutter (minimax-rs_b200/gguf.py) on CPU, and
(GPU) a MoE layer, an attention layer and the LM head loaded from a GGUF file against the same
tensors handed over directly."""
from __future__ import annotations

import importlib

import numpy as np
import pytest

E, H, I = 8, 512, 512
HO = 1024  # the output projection's width: the LM head kernel takes 4, 8, 12 or 16 super-blocks a row


@pytest.fixture(scope="module")
def gguf(pkg):
    return importlib.import_module("minimax_rs_b200.gguf")


def _tensors(synth):
    """A one-layer MiniMax-shaped file: stacked Q4_K gate / up [E][I][H], Q5_K down [E][H][I],
    f32 router and bias, Q8_0 attention (6 query heads, 1 KV head), norms, Q6_K output."""
    qr, kr = 6 * 128, 128
    return {
        "blk.0.ffn_gate_inp.weight": ("F32", (E, H), synth.normal_f32(E * H, 5, 1, 0.02)),
        "blk.0.exp_probs_b.bias": ("F32", (E,), synth.normal_f32(E, 5, 2, 0.01)),
        "blk.0.ffn_gate_exps.weight": ("Q4_K", (E, I, H), synth.kquant(synth.Q4K, 5, 3, E, I, H)),
        "blk.0.ffn_up_exps.weight": ("Q4_K", (E, I, H), synth.kquant(synth.Q4K, 5, 4, E, I, H)),
        "blk.0.ffn_down_exps.weight": ("Q5_K", (E, H, I), synth.kquant(synth.Q5K, 5, 5, E, H, I)),
        "blk.0.attn_q.weight": ("Q8_0", (qr, H), synth.q8_0_blocks(5, 6, qr, H)),
        "blk.0.attn_k.weight": ("Q8_0", (kr, H), synth.q8_0_blocks(5, 7, kr, H)),
        "blk.0.attn_v.weight": ("Q8_0", (kr, H), synth.q8_0_blocks(5, 8, kr, H)),
        "blk.0.attn_output.weight": ("Q8_0", (H, qr), synth.q8_0_blocks(5, 9, H, qr)),
        "blk.0.attn_q_norm.weight": ("F32", (qr,), 1.0 + synth.normal_f32(qr, 5, 10, 0.1)),
        "blk.0.attn_k_norm.weight": ("F32", (kr,), 1.0 + synth.normal_f32(kr, 5, 11, 0.1)),
        "blk.0.attn_norm.weight": ("F16", (H,), (1.0 + synth.normal_f32(H, 5, 12, 0.1)).astype(np.float16)),
        "output_norm.weight": ("F32", (HO,), 1.0 + synth.normal_f32(HO, 5, 13, 0.1)),
        "output.weight": ("Q6_K", (1000, HO), synth.q6k_blocks(5, 14, 1000, HO)),
    }


META = {"general.architecture": "minimax-m2", "minimax-m2.block_count": 1, "minimax-m2.expert_count": E,
        "minimax-m2.rope.freq_base": 5.0e6, "tokenizer.ggml.tokens": ["<s>", "a", "b"], "flag": True,
        "negative": -3}


@pytest.fixture(scope="module")
def gfile(gguf, synth, tmp_path_factory):
    path = tmp_path_factory.mktemp("gguf") / "tiny.gguf"
    t = _tensors(synth)
    gguf.write(path, META, t)
    return gguf.read(path), t


def test_round_trip(gfile):
    g, t = gfile
    assert g.version == 3
    for k, v in META.items():
        got = g.metadata[k]
        assert (abs(got - v) < 1e-6 * abs(v)) if isinstance(v, float) else got == v, k
    assert set(g.tensors) == set(t)
    for name, (tname, shape, data) in t.items():
        ti = g.info(name)
        assert ti.type_name == tname and ti.shape == tuple(shape)
        assert np.array_equal(np.asarray(g.tensor_bytes(name)), np.ascontiguousarray(data).view(np.uint8).reshape(-1))
        assert ti.offset % 32 == 0
    assert np.array_equal(g.array("blk.0.attn_norm.weight"),
                          t["blk.0.attn_norm.weight"][2].astype(np.float32))


def test_tp2_shards_are_slices_of_the_full_tensors(gguf, gfile, synth):
    """TP = 2 (src/tensor_parallel_model.rs:37-61): gate / up rows [r*I/2, (r+1)*I/2) of every
    expert, down K blocks of the same range, Q/K/V rows, output projection K, replicated router."""
    g, t = gfile
    per = I // 2
    for r in range(2):
        shape, gate = gguf.shard_bytes(g, "blk.0.ffn_gate_exps.weight", 2, r)
        assert shape == (E, per, H)
        full = t["blk.0.ffn_gate_exps.weight"][2].reshape(E, I, -1)
        assert np.array_equal(gate, full[:, r * per:(r + 1) * per].reshape(-1))
        # the same window as the synthetic generator's per-rank shard
        assert np.array_equal(gate, synth.kquant(synth.Q4K, 5, 3, E, I, H, row0=r * per, nrows=per).reshape(-1))
        shape, down = gguf.shard_bytes(g, "blk.0.ffn_down_exps.weight", 2, r)
        assert shape == (E, H, per)
        assert np.array_equal(down, synth.kquant(synth.Q5K, 5, 5, E, H, I, kblk0=r * per // 256,
                                                 nkblk=per // 256).reshape(-1))
        shape, q = gguf.shard_bytes(g, "blk.0.attn_q.weight", 2, r)
        fq = t["blk.0.attn_q.weight"][2].reshape(768, -1)
        assert shape == (384, H) and np.array_equal(q, fq[r * 384:(r + 1) * 384].reshape(-1))
        shape, o = gguf.shard_bytes(g, "blk.0.attn_output.weight", 2, r)
        fo = t["blk.0.attn_output.weight"][2].reshape(H, 768 // 32, 34)
        assert shape == (H, 384) and np.array_equal(o, fo[:, r * 12:(r + 1) * 12].reshape(-1))
        shape, rt = gguf.shard_bytes(g, "blk.0.ffn_gate_inp.weight", 2, r)
        assert shape == (E, H) and rt.size == E * H * 4


def test_rejections(gguf, gfile, tmp_path):
    g, _ = gfile
    with pytest.raises(gguf.GGUFError):  # 512 / 4 = 128: not a whole Q5_K block along K
        gguf.shard_bytes(g, "blk.0.ffn_down_exps.weight", 4, 0)
    with pytest.raises(gguf.GGUFError):
        g.info("blk.0.missing.weight")
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"GGML" + bytes(28))
    with pytest.raises(gguf.GGUFError):
        gguf.read(bad)
    short = tmp_path / "short.gguf"
    raw = (gfile[0].path).read_bytes()
    short.write_bytes(raw[:len(raw) - 100])  # last tensor's data cut off
    with pytest.raises(gguf.GGUFError):
        gguf.read(short)


@pytest.mark.gpu
def test_layers_loaded_from_gguf_match_direct_tensors(pkg, gguf, gfile, synth, dev):
    """The MoE layer, the attention layer and the LM head built from
    the file give the same outputs as the same bytes handed over directly."""
    import torch
    g, t = gfile
    T_ = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)  # noqa: E731
    x = T_(synth.normal_f32(H, 5, 20, 1.0).reshape(1, H))
    direct = pkg.MoeLayer(T_(t["blk.0.ffn_gate_inp.weight"][2].reshape(E, H)), T_(t["blk.0.exp_probs_b.bias"][2]),
                          T_(t["blk.0.ffn_gate_exps.weight"][2]), T_(t["blk.0.ffn_up_exps.weight"][2]),
                          T_(t["blk.0.ffn_down_exps.weight"][2]), pkg.Q4K, pkg.Q5K)
    y0 = direct.forward(x).cpu().numpy()
    y1 = gguf.load_moe_layer(pkg, g, 0, dev).forward(x).cpu().numpy()
    assert np.array_equal(y0, y1)
    cos, sin = synth.rope_tables(8, 64)
    a = gguf.load_attn_layer(pkg, g, 0, dev, T_(cos), T_(sin))
    b = pkg.AttnLayer(*(T_(t[f"blk.0.{n}"][2]) for n in ("attn_q.weight", "attn_k.weight", "attn_v.weight",
                                                         "attn_output.weight", "attn_q_norm.weight",
                                                         "attn_k_norm.weight")), T_(cos), T_(sin), H,
                      query_heads=6, kv_heads=1)
    xa = T_(synth.normal_f32(H, 5, 21, 1.0))
    assert np.array_equal(a.forward(xa, 0).cpu().numpy(), b.forward(xa, 0).cpu().numpy())
    h1 = gguf.load_lm_head(pkg, g, dev)
    h2 = pkg.LmHead(T_(t["output.weight"][2]), T_(t["output_norm.weight"][2]), 1000, HO)
    xo = T_(synth.normal_f32(HO, 5, 22, 1.0))
    l1, k1 = h1.forward(xo)
    l2, k2 = h2.forward(xo)
    assert torch.equal(l1, l2) and int(k1.item()) == int(k2.item())
