"""Host forwards of catalog families against transformers' own modules with the same random
weights: BERT and XLM-RoBERTa encoders (final hidden rows and pooled rows, padded batches)."""

import pytest
import torch

transformers = pytest.importorskip("transformers")

from furiosa_opt_models_b200.models import catalog_forward  # noqa: E402


@pytest.mark.parametrize("family", ["bert", "xlm_roberta"])
def test_encoder_matches_transformers(tmp_path, family):
    t = transformers
    kw = dict(hidden_size=64, num_hidden_layers=2, num_attention_heads=4, intermediate_size=128, vocab_size=100,
              max_position_embeddings=40)
    cfg, cls = (t.BertConfig(**kw), t.BertModel) if family == "bert" else (t.XLMRobertaConfig(**kw), t.XLMRobertaModel)
    torch.manual_seed(0)
    model = cls(cfg).eval()
    model.save_pretrained(str(tmp_path))
    ids = torch.randint(3, 100, (2, 9))
    mask = torch.ones_like(ids)
    mask[1, 6:] = 0
    ids[1, 6:] = cfg.pad_token_id
    types = torch.zeros_like(ids)
    if family == "bert":
        types[:, 5:] = 1
    with torch.no_grad():
        want = model(input_ids=ids, attention_mask=mask, token_type_ids=types)
    hidden, pooled = catalog_forward.encoder(str(tmp_path), ids, mask, types)
    real = mask.bool()
    torch.testing.assert_close(hidden[real], want.last_hidden_state[real], rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(pooled, want.pooler_output, rtol=1e-4, atol=1e-4)


def test_encoder_refuses_other_families(tmp_path):
    t = transformers
    cfg = t.MambaConfig(hidden_size=32, num_hidden_layers=1, vocab_size=50, state_size=8)
    t.MambaForCausalLM(cfg).save_pretrained(str(tmp_path))
    with pytest.raises(ValueError, match="not a BERT-style encoder"):
        catalog_forward.encoder(str(tmp_path), torch.zeros(1, 3, dtype=torch.long))


def test_mamba2_recurrence_matches_transformers(tmp_path):
    """The token-by-token selective scan against transformers' chunked scan (its CPU path)."""
    t = transformers
    cfg = t.Mamba2Config(hidden_size=32, num_hidden_layers=2, vocab_size=60, state_size=8, n_groups=2, head_dim=8,
                         num_heads=8, expand=2, chunk_size=4, tie_word_embeddings=False)
    torch.manual_seed(1)
    model = t.Mamba2ForCausalLM(cfg).eval()
    with torch.no_grad():
        for name, prm in model.named_parameters():
            if name.endswith(("A_log", "dt_bias", "D")):
                prm.uniform_(-0.5, 0.5)
    model.save_pretrained(str(tmp_path))
    ids = torch.randint(0, 60, (1, 11))
    with torch.no_grad():
        want = model(input_ids=ids).logits[0]
    got = catalog_forward.mamba2(str(tmp_path), ids[0])
    torch.testing.assert_close(got, want, rtol=2e-4, atol=2e-4)


def test_clip_embeddings_match_transformers(tmp_path):
    t = transformers
    cfg = t.CLIPConfig(text_config=dict(hidden_size=32, intermediate_size=64, num_hidden_layers=2,
                                        num_attention_heads=4, vocab_size=50, max_position_embeddings=12,
                                        eos_token_id=49),
                       vision_config=dict(hidden_size=48, intermediate_size=96, num_hidden_layers=2,
                                          num_attention_heads=4, image_size=16, patch_size=4),
                       projection_dim=24)
    torch.manual_seed(3)
    model = t.CLIPModel(cfg).eval()
    model.save_pretrained(str(tmp_path))
    ids = torch.randint(0, 48, (2, 7))
    ids[:, -1] = 49  # end of text
    pixels = torch.randn(2, 3, 16, 16)
    with torch.no_grad():
        want = model(input_ids=ids, pixel_values=pixels)
    text, image = catalog_forward.clip(str(tmp_path), ids, pixels)
    torch.testing.assert_close(text, want.text_embeds, rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(image, want.image_embeds, rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("ff", ["relu", "gated-gelu"])
def test_t5_encoder_matches_transformers(tmp_path, ff):
    t = transformers
    cfg = t.T5Config(d_model=32, d_kv=8, d_ff=64, num_heads=4, num_layers=2, vocab_size=60, feed_forward_proj=ff,
                     relative_attention_num_buckets=8, relative_attention_max_distance=20)
    torch.manual_seed(4)
    model = t.T5EncoderModel(cfg).eval()
    model.save_pretrained(str(tmp_path))
    ids = torch.randint(0, 60, (2, 30))
    mask = torch.ones_like(ids)
    mask[0, 25:] = 0
    with torch.no_grad():
        want = model(input_ids=ids, attention_mask=mask).last_hidden_state
    got = catalog_forward.t5_encoder(str(tmp_path), ids, mask)
    real = mask.bool()
    torch.testing.assert_close(got[real], want[real], rtol=1e-4, atol=1e-4)


def test_whisper_encoder_matches_transformers(tmp_path):
    t = transformers
    cfg = t.WhisperConfig(d_model=32, encoder_layers=2, decoder_layers=1, encoder_attention_heads=4,
                          decoder_attention_heads=4, encoder_ffn_dim=64, decoder_ffn_dim=64, vocab_size=60,
                          num_mel_bins=16, max_source_positions=20, max_target_positions=10, pad_token_id=0,
                          bos_token_id=1, eos_token_id=2, decoder_start_token_id=1)
    torch.manual_seed(5)
    model = t.WhisperForConditionalGeneration(cfg).eval()
    model.save_pretrained(str(tmp_path))
    features = torch.randn(2, 16, 40)
    with torch.no_grad():
        want = model.model.encoder(features).last_hidden_state
    torch.testing.assert_close(catalog_forward.whisper_encoder(str(tmp_path), features), want, rtol=1e-4, atol=1e-4)


def test_mamba_selective_scan_matches_transformers(tmp_path):
    t = transformers
    cfg = t.MambaConfig(hidden_size=32, num_hidden_layers=2, vocab_size=60, state_size=8, expand=2, conv_kernel=4)
    torch.manual_seed(6)
    model = t.MambaForCausalLM(cfg).eval()
    model.save_pretrained(str(tmp_path))
    ids = torch.randint(0, 60, (1, 9))
    with torch.no_grad():
        want = model(input_ids=ids).logits[0]
    torch.testing.assert_close(catalog_forward.mamba(str(tmp_path), ids[0]), want, rtol=2e-4, atol=2e-4)


def test_bamba_hybrid_matches_transformers(tmp_path):
    """transformers (this version) rotates whole heads whatever partial_rotary_factor says, so the
    checkpoint declares whole-head rotation (attn_rotary_emb = head_dim) for the comparison; the
    prefix rotation of the published configs is checked on its own below."""
    t = transformers
    cfg = t.BambaConfig(hidden_size=32, num_hidden_layers=3, vocab_size=60, num_attention_heads=4, num_key_value_heads=2,
                        intermediate_size=64, attn_layer_indices=[1], mamba_n_heads=8, mamba_d_head=8, mamba_n_groups=2,
                        mamba_d_state=8, mamba_expand=2, mamba_chunk_size=4)
    torch.manual_seed(7)
    model = t.BambaForCausalLM(cfg).eval()
    model.save_pretrained(str(tmp_path))
    import json

    conf = json.loads((tmp_path / "config.json").read_text())
    (tmp_path / "config.json").write_text(json.dumps(dict(conf, attn_rotary_emb=8)))
    ids = torch.randint(0, 60, (1, 10))
    with torch.no_grad():
        want = model(input_ids=ids, use_cache=False).logits[0]
    torch.testing.assert_close(catalog_forward.bamba(str(tmp_path), ids[0]), want, rtol=2e-4, atol=2e-4)


def test_partial_rotation_rotates_the_prefix_only():
    x = torch.randn(6, 2, 8)
    part = catalog_forward._rotate(x, 10000.0, 4)
    assert torch.equal(part[..., 4:], x[..., 4:])
    torch.testing.assert_close(part[..., :4], catalog_forward._rotate(x[..., :4].contiguous(), 10000.0, 4))
    torch.testing.assert_close(part[0], x[0])  # position 0 is not rotated


def test_gemma3_text_matches_transformers(tmp_path):
    t = transformers
    cfg = t.Gemma3TextConfig(hidden_size=32, num_hidden_layers=4, vocab_size=60, num_attention_heads=4,
                             num_key_value_heads=2, head_dim=8, intermediate_size=64, sliding_window=4,
                             layer_types=["sliding_attention", "full_attention"] * 2, max_position_embeddings=64)
    torch.manual_seed(8)
    model = t.Gemma3ForCausalLM(cfg).eval()
    with torch.no_grad():  # norms start at zero scale: give them values
        for name, prm in model.named_parameters():
            if "norm" in name:
                prm.uniform_(-0.5, 0.5)
    model.save_pretrained(str(tmp_path))
    ids = torch.randint(0, 60, (1, 12))
    with torch.no_grad():
        want = model(input_ids=ids, use_cache=False).logits[0]
    torch.testing.assert_close(catalog_forward.gemma3(str(tmp_path), ids[0]), want, rtol=2e-4, atol=2e-4)


@pytest.mark.parametrize("k_eq_v", [False, True])
def test_gemma4_text_matches_transformers(tmp_path, k_eq_v):
    t = transformers
    cfg = t.Gemma4TextConfig(hidden_size=32, num_hidden_layers=4, vocab_size=60, num_attention_heads=4,
                             num_key_value_heads=2, head_dim=8, global_head_dim=16, intermediate_size=64,
                             hidden_size_per_layer_input=8, vocab_size_per_layer_input=30, sliding_window=4,
                             attention_k_eq_v=k_eq_v, num_global_key_value_heads=1 if k_eq_v else None,
                             layer_types=["sliding_attention", "full_attention"] * 2)
    torch.manual_seed(9)
    model = t.Gemma4ForCausalLM(cfg).eval()
    with torch.no_grad():
        for name, prm in model.named_parameters():
            if "norm" in name:
                prm.uniform_(0.5, 1.5)
        for layer in model.model.layers:
            layer.layer_scalar.fill_(0.9)
    model.save_pretrained(str(tmp_path))
    ids = torch.randint(0, 30, (1, 12))
    with torch.no_grad():
        want = model(input_ids=ids, use_cache=False).logits[0]
    torch.testing.assert_close(catalog_forward.gemma4(str(tmp_path), ids[0]), want, rtol=2e-4, atol=2e-4)


@pytest.mark.parametrize("norm_topk", [False, True])
def test_olmoe_matches_transformers(tmp_path, norm_topk):
    t = transformers
    cfg = t.OlmoeConfig(hidden_size=32, num_hidden_layers=2, vocab_size=50, num_attention_heads=4,
                        num_key_value_heads=2, intermediate_size=16, num_experts=4, num_experts_per_tok=2,
                        norm_topk_prob=norm_topk)
    torch.manual_seed(10)
    model = t.OlmoeForCausalLM(cfg).eval()
    model.save_pretrained(str(tmp_path))
    ids = torch.randint(0, 50, (1, 9))
    with torch.no_grad():
        want = model(input_ids=ids, use_cache=False).logits[0]
    torch.testing.assert_close(catalog_forward.olmoe(str(tmp_path), ids[0]), want, rtol=2e-4, atol=2e-4)


# transformers' own group-limited routing does not run in this version, so only greedy routing has
# an oracle here.
@pytest.mark.parametrize(("q_rank", "method"), [(24, "greedy"), (None, "greedy")])
def test_deepseek_v2_matches_transformers(tmp_path, q_rank, method):
    t = transformers
    cfg = t.DeepseekV2Config(hidden_size=32, num_hidden_layers=3, vocab_size=50, num_attention_heads=4,
                             num_key_value_heads=4, intermediate_size=64, moe_intermediate_size=16, n_routed_experts=8,
                             n_shared_experts=2, num_experts_per_tok=2, first_k_dense_replace=1, q_lora_rank=q_rank,
                             kv_lora_rank=16, qk_nope_head_dim=8, qk_rope_head_dim=4, v_head_dim=8, topk_method=method,
                             n_group=4, topk_group=2, routed_scaling_factor=1.5)
    torch.manual_seed(11)
    model = t.DeepseekV2ForCausalLM(cfg).eval()
    model.save_pretrained(str(tmp_path))
    ids = torch.randint(0, 50, (1, 9))
    with torch.no_grad():
        want = model(input_ids=ids, use_cache=False).logits[0]
    torch.testing.assert_close(catalog_forward.deepseek_v2(str(tmp_path), ids[0]), want, rtol=2e-4, atol=2e-4)
