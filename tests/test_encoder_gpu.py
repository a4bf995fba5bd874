"""The Gemma-4 unified media encoder: images (merged patches at their positions) and audio frames
into rows of the text width, against the FP32 PyTorch restatement of the embedders with the same
BF16 roundings; call packing into launches and the refusals of the call."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _load(tmp_path, **widths):
    import furiosa_opt_engine as engine
    from furiosa_opt_models_b200.models import synthetic

    cfg = synthetic.gemma4_unified_config(**widths)
    w = synthetic.write_gemma4_encoder(str(tmp_path / "g4"), cfg)
    device = engine.Device(engine.Placement([0], range(8)))
    enc = engine.LoadOptions().encoder().load(engine.Checkpoint(str(tmp_path / "g4")), device)
    return engine, device, enc, w, cfg


def _hbm(engine, device, t: torch.Tensor):
    return engine.HostTensor.from_dlpack(t.contiguous()).to_hbm(device)


def test_vision_matches_reference(tmp_path):
    from furiosa_opt_models_b200.models import reference

    engine, device, enc, w, cfg = _load(tmp_path)
    assert isinstance(enc, engine.Encoder) and enc.width == 256 and enc.patch_features == 6912
    g = torch.Generator().manual_seed(1)
    images = []
    for n in (5, 37, 1):
        patches = torch.randn(n, 6912, generator=g).bfloat16()
        positions = [[int(torch.randint(0, 40, (1,), generator=g)), int(torch.randint(0, 40, (1,), generator=g))]
                     for _ in range(n)]
        images.append((patches, positions))
    out = enc.vision([engine.vision_language.Image(_hbm(engine, device, p), pos) for p, pos in images])
    assert [tuple(o.shape) for o in out] == [(5, 256), (37, 256), (1, 256)]
    for (p, pos), o in zip(images, out):
        ref = reference.gemma4_vision(w, p, pos)
        got = torch.from_numpy(o.to_host().numpy()).float()
        err = (got - ref).abs().max().item()
        assert err < 3e-2 * max(1.0, ref.abs().max().item()), err


def test_audio_matches_reference_and_packs_launches(tmp_path):
    from furiosa_opt_models_b200.models import reference

    engine, device, enc, w, cfg = _load(tmp_path)
    g = torch.Generator().manual_seed(2)
    # 2000 + 500 frames do not fit one launch of 2304 rows: two launches.
    clips = [torch.randn(n, 640, generator=g).bfloat16() for n in (3, 2000, 500)]
    out = enc.audio([engine.vision_language.Audio(_hbm(engine, device, c)) for c in clips])
    for c, o in zip(clips, out):
        ref = reference.gemma4_audio(w, c)
        got = torch.from_numpy(o.to_host().numpy()).float()
        assert tuple(got.shape) == (c.shape[0], 256)
        assert (got - ref).abs().max().item() < 3e-2 * max(1.0, ref.abs().max().item())


def test_call_refusals(tmp_path):
    engine, device, enc, w, cfg = _load(tmp_path)
    ok = _hbm(engine, device, torch.zeros(2, 6912).bfloat16())
    with pytest.raises(ValueError, match="reaches past the 40 positions"):
        enc.vision([engine.vision_language.Image(ok, [[0, 0], [40, 1]])])
    with pytest.raises(ValueError, match="a patch position is negative"):
        enc.vision([engine.vision_language.Image(ok, [[0, 0], [-1, 1]])])
    with pytest.raises(ValueError, match="one for each position"):
        engine.vision_language.Image(ok, [[0, 0]])
    wide = _hbm(engine, device, torch.zeros(2, 640).bfloat16())
    with pytest.raises(ValueError, match="do not hold 2 rows of 6912 BF16 values"):
        enc.vision([engine.vision_language.Image(wide, [[0, 0], [1, 1]])])
    big = _hbm(engine, device, torch.zeros(2305, 640).bfloat16())
    with pytest.raises(NotImplementedError, match="item 0 holds 2305 rows; a launch takes at most 2304"):
        enc.audio([engine.vision_language.Audio(big)])


def test_vllm_media_step_matches_the_encoder(tmp_path):
    """The vLLM encoder-only step (furiosa_opt_vllm.media) on the real encoder: an image with the
    processor's padding patches and an audio clip with padded frames give the rows of the encoder
    called on the valid patches and frames alone."""
    from types import SimpleNamespace as ns

    from furiosa_opt_vllm import media

    engine, device, enc, w, cfg = _load(tmp_path)
    g = torch.Generator().manual_seed(3)
    pix = torch.randn(6, 6912, generator=g).bfloat16()
    pos = torch.tensor([[0, 0], [1, 0], [2, 1], [3, 1], [-1, -1], [-1, -1]])
    frames = torch.randn(9, 640, generator=g).bfloat16()
    mask = torch.tensor([1] * 7 + [0] * 2)
    image = ns(identifier="i", modality="image", data={"pixel_values": pix, "pixel_position_ids": pos},
               mm_position=ns(get_num_embeds=lambda: 4))
    audio = ns(identifier="a", modality="audio", data={"input_features_padded": frames, "input_features_mask": mask},
               mm_position=ns(get_num_embeds=lambda: 7))
    m = media.Media(engine, enc, device)
    so = ns(finished_req_ids=set(), free_encoder_mm_hashes=[], scheduled_new_reqs=[ns(req_id="r", mm_features=[image, audio])],
            scheduled_encoder_inputs={"r": [0, 1]})
    assert m.step(so) == ["i", "a"]
    (want_i,) = enc.vision([engine.vision_language.Image(_hbm(engine, device, pix[:4]), pos[:4].tolist())])
    (want_a,) = enc.audio([engine.vision_language.Audio(_hbm(engine, device, frames[:7]))])
    assert torch.equal(m.host["i"].float(), torch.from_numpy(want_i.to_host().numpy()))
    assert torch.equal(m.host["a"].float(), torch.from_numpy(want_a.to_host().numpy()))
