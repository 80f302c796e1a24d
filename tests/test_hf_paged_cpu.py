"""Host-side logic of the Hugging Face adapter (no kernel is launched)."""
import pytest
import torch

from conftest import load_pkg


def _cfg(**kw):
    from transformers import Lfm2Config
    from oracle import lfm2_attention as orc
    base = dict(hidden_size=1024, intermediate_size=3840, num_hidden_layers=14, num_attention_heads=16,
                num_key_value_heads=8, vocab_size=65536, layer_types=list(orc.LFM25_LAYER_TYPES))
    base.update(kw)
    return Lfm2Config(**base)


def test_paged_cache_layers_and_lengths():
    hf = load_pkg("hf_paged")
    cfg = _cfg()
    cache = hf.B200PagedCache(cfg, max_batch_size=2, max_cache_len=100, device="cpu")
    att = [i for i, t in enumerate(cfg.layer_types) if t == "full_attention"]
    assert [type(cache.layers[i]).__name__ for i in att] == ["PagedAttentionLayer"] * len(att)
    assert cache.pool.num_layers == len(att) and cache.tables.shape == (2, 2)
    assert cache.get_seq_length() == 0
    k = torch.zeros(2, 8, 5, 64, dtype=torch.bfloat16)
    kk, vv = cache.update(k, k, att[0])
    assert kk is k and vv is k
    assert cache.get_seq_length() == 5 and cache.get_mask_sizes(1, att[0]) == (6, 0)
    with pytest.raises(ValueError, match="capacity"):
        cache.update(torch.zeros(2, 8, 96, 64, dtype=torch.bfloat16), torch.zeros(2, 8, 96, 64,
                     dtype=torch.bfloat16), att[0])
    with pytest.raises(ValueError, match="batch"):
        cache.update(torch.zeros(3, 8, 1, 64, dtype=torch.bfloat16), torch.zeros(3, 8, 1, 64,
                     dtype=torch.bfloat16), att[1])
    cache.crop(2)
    assert cache.get_seq_length() == 2
    cache.reset()
    assert cache.get_seq_length() == 0


def test_attention_without_cache_is_rejected():
    hf = load_pkg("hf_paged")

    class M:
        layer_idx = 2
    q = torch.zeros(1, 16, 1, 64, dtype=torch.bfloat16)
    k = torch.zeros(1, 8, 1, 64, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="B200PagedCache"):
        hf.paged_attention(M(), q, k, k, None)


def test_wrong_head_shape_is_rejected():
    hf = load_pkg("hf_paged")
    with pytest.raises(ValueError, match="16 query heads"):
        hf.B200PagedCache(_cfg(num_attention_heads=8, num_key_value_heads=8), max_batch_size=1,
                          max_cache_len=64, device="cpu")


def test_register_adds_the_implementation():
    from transformers import AttentionInterface
    hf = load_pkg("hf_paged")
    hf.register()
    assert AttentionInterface._global_mapping["b200_paged"] is hf.paged_attention
