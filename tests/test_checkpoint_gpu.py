"""MLX-format safetensors checkpoints into the engine (load_weights_from_manifest,
crates/serve/src/loader/weights.rs:17-284).

A model made from seeded weights is written out tensor by tensor under the
MLX checkpoint names (uint32 codes, bf16 scales / biases / norms), loaded into
a second model through emx_qwen3_load_safetensors, and must hold the same
bytes and produce the same logits bits and greedy tokens.  The shipped-fused
layout (qkv_proj / gate_up_proj, preferred by the reference when present), a
sharded checkpoint with an index file, and the loader's refusals are covered
too.
"""
import json
import os

import numpy as np
import pytest

import emx

pytestmark = pytest.mark.gpu

DENSE = dict(hidden=512, layers=2, n_q=8, n_kv=2, inter=1024, vocab=2048, kv_cap=128, max_prefill=32)
MOE = dict(hidden=512, layers=2, n_q=8, n_kv=2, inter=1024, vocab=2048, tied=False, n_experts=16, top_k=4,
           moe_inter=256, kv_cap=128, max_prefill=32)
PROMPT = np.array([5, 17, 300, 42, 1000, 7, 99, 2047], dtype=np.int32)


@pytest.fixture(scope="module")
def ctx():
    c = emx.Ctx(0)
    yield c
    c.close()


def dump(m):
    """name -> array of every tensor the model takes (full MLX shapes)."""
    out = {}
    for name in m.tensor_names():
        shape, dt = m.tensor_shape(name)
        n = int(np.prod(shape)) * np.dtype(dt).itemsize
        out[name] = np.frombuffer(m.read_tensor(name, n), dtype=dt).reshape(shape)
    return out


def run(m):
    m.reset()
    tok, logits = m.prefill(PROMPT, want_logits=True)
    res = [(tok, logits)]
    for _ in range(4):
        tok, logits = m.decode_step(tok, want_logits=True)
        res.append((tok, logits))
    return res


def same_model(a, b):
    da, db = dump(a), dump(b)
    assert sorted(da) == sorted(db)
    for k in da:
        assert np.array_equal(da[k], db[k]), k
    for (ta, la), (tb, lb) in zip(run(a), run(b)):
        assert ta == tb
        assert np.array_equal(la, lb)


@pytest.mark.parametrize("kw", [DENSE, MOE], ids=["dense", "moe"])
def test_round_trip_through_a_checkpoint_directory(ctx, tmp_path, kw):
    cfg = emx.Qwen3Config(**kw)
    a = emx.Qwen3(ctx, cfg)
    a.init_random(11)
    tensors = dump(a)
    tensors["model.layers.0.mlp.extra_buffer"] = np.zeros(4, np.uint16)  # off the path: skipped
    emx.write_safetensors(str(tmp_path / "model.safetensors"), tensors, {"format": "mlx"})
    b = emx.Qwen3(ctx, cfg)
    n = b.load_safetensors(str(tmp_path))
    assert n == len(tensors) - 1
    same_model(a, b)
    a.close()
    b.close()


def test_shipped_fused_projections_and_sharded_index(ctx, tmp_path):
    cfg = emx.Qwen3Config(**DENSE)
    a = emx.Qwen3(ctx, cfg)
    a.init_random(12)
    t = dump(a)
    fused = {}
    for l in range(cfg.layers):
        p = f"model.layers.{l}."
        for part in ("weight", "scales", "biases"):
            fused[p + f"self_attn.qkv_proj.{part}"] = np.concatenate(
                [t.pop(p + f"self_attn.{x}_proj.{part}") for x in "qkv"], axis=0)
            fused[p + f"mlp.gate_up_proj.{part}"] = np.concatenate(
                [t.pop(p + f"mlp.{x}_proj.{part}") for x in ("gate", "up")], axis=0)
    t.update(fused)
    # model_fused.safetensors is preferred over a (here broken) model.safetensors
    d1 = tmp_path / "fused"
    d1.mkdir()
    emx.write_safetensors(str(d1 / "model_fused.safetensors"), t)
    open(d1 / "model.safetensors", "wb").write(b"\x00")
    b = emx.Qwen3(ctx, cfg)
    b.load_safetensors(str(d1))
    same_model(a, b)
    # the same tensors split over two shard files named by an index
    d2 = tmp_path / "sharded"
    d2.mkdir()
    names = sorted(t)
    halves = {"model-00001-of-00002.safetensors": names[: len(names) // 2],
              "model-00002-of-00002.safetensors": names[len(names) // 2:]}
    wmap = {}
    for fn, ns in halves.items():
        emx.write_safetensors(str(d2 / fn), {k: t[k] for k in ns})
        wmap.update({k: fn for k in ns})
    json.dump({"metadata": {}, "weight_map": wmap}, open(d2 / "model.safetensors.index.json", "w"))
    c = emx.Qwen3(ctx, cfg)
    c.load_safetensors(str(d2))
    same_model(a, c)
    for m in (a, b, c):
        m.close()


def test_loader_refusals(ctx, tmp_path):
    cfg = emx.Qwen3Config(**DENSE)
    a = emx.Qwen3(ctx, cfg)
    a.init_random(13)
    t = dump(a)
    b = emx.Qwen3(ctx, cfg)

    def attempt(tensors, what):
        p = str(tmp_path / f"{what}.safetensors")
        emx.write_safetensors(p, tensors)
        with pytest.raises(emx.EmxError) as ei:
            b.load_safetensors(p)
        return ei.value.msg

    missing = dict(t)
    del missing["model.layers.1.self_attn.k_norm.weight"]
    assert "missing model.layers.1.self_attn.k_norm.weight" in attempt(missing, "missing")
    wrong = dict(t)
    wrong["model.norm.weight"] = ("F32", t["model.norm.weight"].astype(np.float32))
    assert "F32" in attempt(wrong, "dtype")
    transposed = dict(t)
    w = t["model.layers.0.self_attn.o_proj.scales"]
    transposed["model.layers.0.self_attn.o_proj.scales"] = np.ascontiguousarray(w.reshape(w.shape[::-1]))
    assert "shape" in attempt(transposed, "shape")
    untied = dict(t)
    for part in ("weight", "scales", "biases"):
        untied[f"lm_head.{part}"] = t[f"model.embed_tokens.{part}"]
    assert "tied" in attempt(untied, "untied")
    with pytest.raises(emx.EmxError) as ei:
        b.load_safetensors(str(tmp_path / "no_such_dir_or_file"))
    assert "cannot open" in ei.value.msg
    empty = tmp_path / "emptydir"
    empty.mkdir()
    with pytest.raises(emx.EmxError) as ei:
        b.load_safetensors(str(empty))
    assert "model.safetensors not found" in ei.value.msg
    a.close()
    b.close()


def test_model_from_a_directory_with_config_json(ctx, tmp_path):
    """Qwen3.from_dir: config.json (emx_qwen3_config_from_dir) then the
    checkpoint; the model equals the one that wrote them."""
    cfg = emx.Qwen3Config(**DENSE)
    a = emx.Qwen3(ctx, cfg)
    a.init_random(14)
    emx.write_safetensors(str(tmp_path / "model.safetensors"), dump(a))
    conf = {"hidden_size": cfg.hidden, "num_hidden_layers": cfg.layers, "intermediate_size": cfg.inter,
            "num_attention_heads": cfg.n_q, "num_key_value_heads": cfg.n_kv, "head_dim": cfg.head_dim,
            "vocab_size": cfg.vocab, "tie_word_embeddings": True, "quantization": {"group_size": 64, "bits": 4}}
    (tmp_path / "config.json").write_text(json.dumps(conf))
    b = emx.Qwen3.from_dir(ctx, str(tmp_path), kv_cap=cfg.kv_cap, max_prefill=cfg.max_prefill)
    same_model(a, b)
    a.close()
    b.close()
