"""The DDIM sampler of a diffusion pipeline's scheduler config (`scheduler/scheduler_config.json`).

A schedule of `num_train_timesteps` noise levels: betas (linear, scaled-linear, the cosine
"squaredcos_cap_v2" schedule of Nichol and Dhariwal 2021, or the config's trained betas), their
cumulative products of 1 - beta in FP32, and optionally Lin et al. 2023's rescale to zero terminal
SNR. `timesteps(n)` picks n of the training timesteps (leading, trailing or linspace spacing, with
the config's offset); `step` is the DDIM update of Song et al. 2021 (eq. 12) from the model's
epsilon, v or sample prediction, with optional clipping of the predicted sample and `eta` of
stochasticity. The reference parses the same config for its DiT pipeline
(crates/furiosa-opt-models/src/models/config/ddim.rs); the key names are diffusers' public
scheduler-config format.
"""

from __future__ import annotations

import dataclasses
import math

import numpy as np

PREDICTIONS = ("epsilon", "v_prediction", "sample")
SPACINGS = ("leading", "trailing", "linspace")


def _cosine_betas(count: int, max_beta: float = 0.999) -> np.ndarray:
    """Nichol and Dhariwal's schedule: alpha_bar(t) = cos((t + 0.008) / 1.008 * pi / 2)^2 over
    t in [0, 1], beta_i = 1 - alpha_bar((i + 1) / T) / alpha_bar(i / T), capped at `max_beta`."""

    def alpha_bar(t: float) -> float:
        return math.cos((t + 0.008) / 1.008 * math.pi / 2) ** 2

    return np.array([min(1 - alpha_bar((i + 1) / count) / alpha_bar(i / count), max_beta) for i in range(count)],
                    dtype=np.float32)


def _zero_terminal_snr(betas: np.ndarray) -> np.ndarray:
    """Lin et al. 2023, algorithm 1: shift and scale sqrt(alpha_bar) so that the last timestep has
    zero signal and the first keeps its value, then recover the betas."""
    root = np.sqrt(np.cumprod(1.0 - betas.astype(np.float64)))
    first, last = root[0], root[-1]
    root = (root - last) * first / (first - last)
    bar = root**2
    alphas = np.concatenate([bar[:1], bar[1:] / bar[:-1]])
    return (1.0 - alphas).astype(np.float32)


@dataclasses.dataclass(frozen=True)
class Schedule:
    alphas_cumprod: np.ndarray  # FP32 [num_train_timesteps]
    final_alpha_cumprod: float  # the alpha_bar a step to before timestep 0 lands on
    prediction: str = "epsilon"
    spacing: str = "leading"
    offset: int = 0
    clip: float | None = None  # the predicted sample's clipping range, when clipped

    @property
    def count(self) -> int:
        return len(self.alphas_cumprod)

    @classmethod
    def from_config(cls, cfg: dict) -> "Schedule":
        """Parses a scheduler config, refusing (ValueError naming the key) what DDIM does not run."""
        count = int(cfg.get("num_train_timesteps", 1000))
        if count <= 0:
            raise ValueError("num_train_timesteps: a schedule has at least one timestep")
        prediction = cfg.get("prediction_type") or "epsilon"
        if prediction not in PREDICTIONS:
            raise ValueError(f"prediction_type: {prediction}, DDIM steps from {', '.join(PREDICTIONS)}")
        if cfg.get("thresholding"):
            raise ValueError("thresholding: dynamic thresholding of the predicted sample is not served")
        spacing = cfg.get("timestep_spacing") or "leading"
        if spacing not in SPACINGS:
            raise ValueError(f"timestep_spacing: {spacing}, one of {', '.join(SPACINGS)}")
        trained = cfg.get("trained_betas")
        if trained is not None:
            betas = np.asarray(trained, dtype=np.float32)
            if betas.shape != (count,):
                raise ValueError(f"trained_betas: {betas.size} betas for {count} timesteps")
        else:
            start, end = float(cfg.get("beta_start", 0.0001)), float(cfg.get("beta_end", 0.02))
            if not (math.isfinite(start) and math.isfinite(end)):
                raise ValueError("beta_start, beta_end: finite numbers")
            kind = cfg.get("beta_schedule") or "linear"
            if kind == "linear":
                betas = np.linspace(start, end, count, dtype=np.float32)
            elif kind == "scaled_linear":
                betas = np.linspace(start**0.5, end**0.5, count, dtype=np.float32) ** 2
            elif kind == "squaredcos_cap_v2":
                betas = _cosine_betas(count)
            else:
                raise ValueError(f"beta_schedule: {kind}, one of linear, scaled_linear, squaredcos_cap_v2")
        if cfg.get("rescale_betas_zero_snr"):
            betas = _zero_terminal_snr(betas)
        if not ((betas >= 0) & (betas <= 1)).all():
            raise ValueError("betas: each in [0, 1]")
        alphas_cumprod = np.cumprod((1.0 - betas).astype(np.float32), dtype=np.float32)
        final = 1.0 if cfg.get("set_alpha_to_one", True) else float(alphas_cumprod[0])
        clip = float(cfg.get("clip_sample_range", 1.0)) if cfg.get("clip_sample", True) else None
        return cls(alphas_cumprod, final, prediction, spacing, int(cfg.get("steps_offset", 0)), clip)

    def timesteps(self, n: int) -> np.ndarray:
        """The `n` training timesteps a sampling run visits, from the noisiest."""
        if not 0 < n <= self.count:
            raise ValueError(f"num_inference_steps: {n}, between 1 and {self.count}")
        if self.spacing == "leading":
            t = (np.arange(n) * (self.count // n)).round()[::-1] + self.offset
        elif self.spacing == "trailing":
            t = np.round(np.arange(self.count, 0, -self.count / n)) - 1
        else:
            t = np.linspace(0, self.count - 1, n).round()[::-1]
        return t.astype(np.int64).copy()

    def step(self, model_output, t: int, sample, n: int, eta: float = 0.0, noise=None):
        """The sample at the previous timestep of an `n`-step run (DDIM, Song et al. 2021 eq. 12):
        the predicted clean sample re-noised to the previous level along the predicted noise, with
        `eta` times the DDPM posterior's standard deviation of fresh `noise`. Works on torch tensors
        (any device) or numpy arrays."""
        prev = t - self.count // n
        a = float(self.alphas_cumprod[t])
        a_prev = float(self.alphas_cumprod[prev]) if prev >= 0 else self.final_alpha_cumprod
        b = 1.0 - a
        if self.prediction == "epsilon":
            x0 = (sample - b**0.5 * model_output) / a**0.5
            eps = model_output
        elif self.prediction == "v_prediction":
            x0 = a**0.5 * sample - b**0.5 * model_output
            eps = a**0.5 * model_output + b**0.5 * sample
        else:
            x0 = model_output
            eps = (sample - a**0.5 * x0) / b**0.5
        if self.clip is not None:
            x0 = x0.clip(-self.clip, self.clip)
        var = (1 - a_prev) / b * (1 - a / a_prev) if b > 0 else 0.0
        std = eta * max(var, 0.0) ** 0.5
        out = a_prev**0.5 * x0 + max(1 - a_prev - std**2, 0.0) ** 0.5 * eps
        if std > 0:
            if noise is None:
                raise ValueError("eta > 0 draws noise: pass `noise` of the sample's shape")
            out = out + std * noise
        return out
