"""The DDIM sampler of a scheduler config: betas and FP32 cumulative alphas against their closed
forms, timestep spacings, and the update, whose deterministic run from an oracle noise prediction
lands on the clean sample."""

import math

import numpy as np
import pytest
import torch

from furiosa_opt_models_b200.models.ddim import Schedule

SD = {"_class_name": "DDIMScheduler", "beta_start": 0.00085, "beta_end": 0.012, "beta_schedule": "scaled_linear",
      "clip_sample": False, "num_train_timesteps": 1000, "set_alpha_to_one": False, "steps_offset": 1}


def test_alphas_follow_the_beta_schedules():
    s = Schedule.from_config({"beta_schedule": "linear"})
    betas = np.linspace(0.0001, 0.02, 1000)
    want = np.cumprod(1 - betas)
    assert s.alphas_cumprod.dtype == np.float32
    np.testing.assert_allclose(s.alphas_cumprod, want, rtol=2e-5)
    s = Schedule.from_config(SD)
    betas = np.linspace(math.sqrt(0.00085), math.sqrt(0.012), 1000) ** 2
    np.testing.assert_allclose(s.alphas_cumprod, np.cumprod(1 - betas), rtol=2e-5)
    assert s.final_alpha_cumprod == pytest.approx(1 - 0.00085, rel=1e-6)  # set_alpha_to_one false
    cos = Schedule.from_config({"beta_schedule": "squaredcos_cap_v2"})
    bar = [math.cos((t / 1000 + 0.008) / 1.008 * math.pi / 2) ** 2 / math.cos(0.008 / 1.008 * math.pi / 2) ** 2
           for t in range(1, 1001)]
    np.testing.assert_allclose(cos.alphas_cumprod[:900], bar[:900], rtol=1e-4)
    trained = Schedule.from_config({"num_train_timesteps": 3, "trained_betas": [0.1, 0.2, 0.5]})
    np.testing.assert_allclose(trained.alphas_cumprod, [0.9, 0.72, 0.36], rtol=1e-6)


def test_zero_terminal_snr_rescale():
    s = Schedule.from_config(dict(SD, rescale_betas_zero_snr=True))
    plain = Schedule.from_config(SD)
    assert s.alphas_cumprod[-1] == pytest.approx(0.0, abs=1e-7)
    assert s.alphas_cumprod[0] == pytest.approx(plain.alphas_cumprod[0], rel=1e-5)
    assert (np.diff(s.alphas_cumprod) < 0).all()


@pytest.mark.parametrize(("spacing", "want"), [
    ("leading", [901, 801, 701, 601, 501, 401, 301, 201, 101, 1]),
    ("trailing", [999, 899, 799, 699, 599, 499, 399, 299, 199, 99]),
    ("linspace", [999, 888, 777, 666, 555, 444, 333, 222, 111, 0])])
def test_timestep_spacings(spacing, want):
    s = Schedule.from_config(dict(SD, timestep_spacing=spacing, steps_offset=1 if spacing == "leading" else 0))
    assert s.timesteps(10).tolist() == want


@pytest.mark.parametrize("prediction", ["epsilon", "v_prediction", "sample"])
def test_deterministic_run_from_an_oracle_lands_on_the_clean_sample(prediction):
    """x_t = sqrt(a) x0 + sqrt(1 - a) eps for a fixed (x0, eps): a model that predicts exactly that
    eps (or v, or x0) takes a 25-step eta=0 run from pure-ish noise to x0."""
    s = Schedule.from_config(dict(SD, prediction_type=prediction, set_alpha_to_one=True, steps_offset=0))
    g = torch.Generator().manual_seed(0)
    x0 = torch.randn(4, 8, generator=g, dtype=torch.float64)
    eps = torch.randn(4, 8, generator=g, dtype=torch.float64)
    n = 25
    ts = s.timesteps(n)
    a0 = float(s.alphas_cumprod[ts[0]])
    x = a0**0.5 * x0 + (1 - a0) ** 0.5 * eps
    for t in ts:
        a = float(s.alphas_cumprod[t])
        out = {"epsilon": eps, "v_prediction": a**0.5 * eps - (1 - a) ** 0.5 * x0, "sample": x0}[prediction]
        x = s.step(out, int(t), x, n)
    torch.testing.assert_close(x, x0, rtol=1e-9, atol=1e-9)


def test_stochastic_steps_add_the_posterior_noise():
    s = Schedule.from_config(dict(SD, clip_sample=False))
    x = torch.ones(3)
    eps = torch.zeros(3)
    noise = torch.full((3,), 2.0)
    det = s.step(eps, 501, x, 10)
    sto = s.step(eps, 501, x, 10, eta=1.0, noise=noise)
    a, a_prev = float(s.alphas_cumprod[501]), float(s.alphas_cumprod[401])
    std = ((1 - a_prev) / (1 - a) * (1 - a / a_prev)) ** 0.5
    torch.testing.assert_close(det, (a_prev / a) ** 0.5 * x)  # no predicted noise: the clean sample re-scaled
    torch.testing.assert_close(sto - det, std * noise, rtol=1e-5, atol=1e-6)
    with pytest.raises(ValueError, match="noise"):
        s.step(eps, 501, x, 10, eta=1.0)


def test_clipping_bounds_the_predicted_sample():
    s = Schedule.from_config({"clip_sample": True, "clip_sample_range": 1.0, "set_alpha_to_one": True})
    x = np.full(2, 50.0)
    out = s.step(np.zeros(2), 0, x, 1000)  # the last step returns the (clipped) clean sample
    np.testing.assert_allclose(out, [1.0, 1.0])


@pytest.mark.parametrize(("cfg", "key"), [({"prediction_type": "flow"}, "prediction_type"),
                                          ({"thresholding": True}, "thresholding"),
                                          ({"beta_schedule": "sigmoid"}, "beta_schedule"),
                                          ({"num_train_timesteps": 3, "trained_betas": [0.1]}, "trained_betas"),
                                          ({"timestep_spacing": "karras"}, "timestep_spacing"),
                                          ({"num_train_timesteps": 0}, "num_train_timesteps")])
def test_refusals_name_the_key(cfg, key):
    with pytest.raises(ValueError, match=key):
        Schedule.from_config(cfg)
    with pytest.raises(ValueError, match="num_inference_steps"):
        Schedule.from_config(SD).timesteps(1001)
