"""config.json -> emx_qwen3_config (Qwen3Config::from_dir,
crates/serve/src/config.rs:6-91), host only: the serde defaults, head_dim from
hidden / heads when absent, MLX's model-wide and per-module quantization, the
MoE keys, and the refusals."""
import json
import os

import pytest

import emx


def write(tmp_path, cfg):
    d = tmp_path / "model"
    d.mkdir(exist_ok=True)
    (d / "config.json").write_text(json.dumps(cfg))
    return str(d)


QWEN3_1_7B = {
    "architectures": ["Qwen3ForCausalLM"], "hidden_size": 2048, "num_hidden_layers": 28,
    "intermediate_size": 6144, "num_attention_heads": 16, "num_key_value_heads": 8, "head_dim": 128,
    "vocab_size": 151936, "rms_norm_eps": 1e-6, "rope_theta": 1000000, "tie_word_embeddings": True,
    "quantization": {"group_size": 64, "bits": 4},
}


def test_mixed_precision_dense_config_is_the_c3_shape(tmp_path):
    cfg = dict(QWEN3_1_7B)
    q = {"group_size": 64, "bits": 4}
    for l in range(28):
        for p in ("q_proj", "k_proj", "v_proj", "o_proj"):
            q[f"model.layers.{l}.self_attn.{p}"] = {"group_size": 64, "bits": 8}
    cfg["quantization"] = q
    got = emx.Qwen3Config.from_dir(write(tmp_path, cfg), kv_cap=16384, max_prefill=8192)
    want = emx.CONFIGS["c3"]
    for f in ("hidden", "layers", "n_q", "n_kv", "head_dim", "inter", "vocab", "tied", "attn_bits", "attn_group",
              "mlp_bits", "mlp_group", "embed_bits", "lm_bits", "n_experts", "kv_cap"):
        assert getattr(got, f) == getattr(want, f), f
    assert got.eps == pytest.approx(1e-6) and got.rope_theta == 1e6


def test_defaults_follow_the_reference(tmp_path):
    cfg = {k: v for k, v in QWEN3_1_7B.items() if k not in ("head_dim", "rms_norm_eps", "rope_theta",
                                                               "tie_word_embeddings")}
    got = emx.Qwen3Config.from_dir(os.path.join(write(tmp_path, cfg), "config.json"))
    assert got.head_dim == 2048 // 16 and got.norm_groups == 1 and got.tied
    assert got.eps == pytest.approx(1e-6) and got.rope_theta == 1e6


def test_moe_config(tmp_path):
    cfg = {"hidden_size": 2048, "num_hidden_layers": 48, "intermediate_size": 6144, "num_attention_heads": 32,
           "num_key_value_heads": 4, "head_dim": 128, "vocab_size": 151936, "tie_word_embeddings": False,
           "num_experts": 128, "num_experts_per_tok": 8, "moe_intermediate_size": 768, "norm_topk_prob": True,
           "quantization": {"group_size": 64, "bits": 4, "mode": "affine",
                            "model.layers.0.mlp.gate": {"group_size": 64, "bits": 8}}}
    got = emx.Qwen3Config.from_dir(write(tmp_path, cfg))
    assert (got.n_experts, got.top_k, got.moe_inter, got.norm_topk, got.tied) == (128, 8, 768, True, False)
    assert got.router_bits == 8 and got.expert_bits == 4 and got.attn_bits == 4


@pytest.mark.parametrize("edit,words", [
    (lambda c: c.pop("hidden_size"), "hidden_size"),
    (lambda c: c.pop("quantization"), "quantization"),
    (lambda c: c["quantization"].update({"model.layers.0.mlp.down_proj": False}), "not quantized"),
    (lambda c: c["quantization"].update({"model.layers.0.self_attn.q_proj": {"group_size": 64, "bits": 8},
                                         "model.layers.1.self_attn.q_proj": {"group_size": 32, "bits": 8}}),
     "one setting per kind"),
    (lambda c: c.update({"num_experts": 8, "num_experts_per_tok": 0}), "num_experts_per_tok"),
    (lambda c: c.update({"rope_theta": "big"}), "rope_theta"),
])
def test_refusals(tmp_path, edit, words):
    cfg = json.loads(json.dumps(QWEN3_1_7B))
    edit(cfg)
    with pytest.raises(emx.EmxError) as ei:
        emx.Qwen3Config.from_dir(write(tmp_path, cfg))
    assert ei.value.code == emx.ERR_INVALID and words in ei.value.msg


def test_missing_config_and_bad_sizes(tmp_path):
    with pytest.raises(emx.EmxError):
        emx.Qwen3Config.from_dir(str(tmp_path))
    with pytest.raises(emx.EmxError):
        emx.Qwen3Config.from_dir(write(tmp_path, QWEN3_1_7B), kv_cap=64, max_prefill=128)
