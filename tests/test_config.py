"""Host-side manifest rules: a restatement of config.go:84-232."""

import pytest

from rembed_b200.config import Config, ConfigError
from rembed_b200 import synth


def base(**kw):
    c = dict(name="t", model_type="bert", hidden_size=64, num_hidden_layers=1, num_attention_heads=2,
             intermediate_size=128, vocab_size=100, max_position_embeddings=32, pooling="mean")
    c.update(kw)
    return Config(**c)


def test_presets_validate():
    for name in synth.PRESETS:
        synth.preset(name)


def test_eps_default():  # config.go:228-230
    assert base().validate().layer_norm_eps == pytest.approx(1e-12)


@pytest.mark.parametrize("kw,frag", [
    (dict(hidden_size=0), "non-positive"),
    (dict(num_attention_heads=3), "not divisible"),
    (dict(pooling="max"), "pooling"),
    (dict(tokenizer="bpe"), "tokenizer"),
    (dict(model_type="gpt2"), "unsupported"),
    (dict(model_type="roberta", pad_token_id=0), "pad_token_id >= 1"),
    (dict(model_type="mpnet", relative_attention_num_buckets=16, pad_token_id=1), "hardcodes 32"),
    (dict(model_type="mpnet", relative_attention_num_buckets=32, pad_token_id=2), "padding_idx=1"),
    (dict(model_type="modernbert"), "global_attn_every_n_layers"),
    (dict(model_type="qwen3", head_dim=3), "even head_dim"),
    (dict(model_type="gemma3", head_dim=64, num_key_value_heads=1), "sliding_window"),
    (dict(model_type="nomic_bert", head_dim=16, rope_theta=1.0), "must equal hidden_size"),
])
def test_validate_refuses(kw, frag):
    with pytest.raises(ConfigError, match=frag):
        base(**kw).validate()


def test_position_offset_and_max_seq_len():  # config.go:84-95
    c = base(model_type="roberta", pad_token_id=1, max_position_embeddings=514).validate()
    assert c.position_offset() == 2 and c.max_seq_len() == 512
    assert base().validate().position_offset() == 0


def test_manifest_round_trip(tmp_path):
    cfg = synth.preset("tiny-bert")
    p = tmp_path / "manifest.json"
    p.write_text(cfg.to_json())
    back = Config.load(p)
    assert back.hidden_size == cfg.hidden_size and back.pooling == cfg.pooling


def test_safetensors_round_trip(tmp_path):
    import numpy as np

    cfg = synth.preset("tiny-bert")
    w = synth.make_weights(cfg, seed=3)
    synth.write_model_dir(tmp_path / "m", cfg, w)
    back = synth.read_safetensors(tmp_path / "m" / "model.safetensors")
    assert set(back) == set(w)
    for k in w:
        assert np.array_equal(back[k], w[k])


def test_pack_and_batch():
    import numpy as np
    from rembed_b200.embedder import pack

    ids, cu = pack([[1, 2, 3], [4], [5, 6]])
    assert ids.tolist() == [1, 2, 3, 4, 5, 6] and cu.tolist() == [0, 3, 4, 6]
    cfg = synth.preset("bge-base")
    ids, cu = synth.make_batch(cfg, 8, 16, 64, seed=2)
    lens = np.diff(cu)
    assert lens.min() >= 16 and lens.max() <= 64 and ids.shape[0] == cu[-1]
    assert np.all(ids[cu[:-1]] == 101) and np.all(ids[cu[1:] - 1] == 102)
