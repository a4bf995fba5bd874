"""A vision-language checkpoint's media encoder served as vLLM's encoder-only instance.

vLLM's disaggregated encoding runs the media encoder in its own instance: each step's scheduler
output names the media items to embed (`scheduled_encoder_inputs`), the instance embeds them and
hands the rows to the encoder-cache connector (`ECConnectorModelRunnerMixin`), from which another
instance's language model reads them; a hash vLLM frees (`free_encoder_mm_hashes`) is dropped. No
token is sampled: the step's output is vLLM's empty encoder output, which finishes each request
once its items are embedded.

The engine's `Encoder` embeds images and video frames as merged patches at their (x, y) positions
and audio as frame rows; the processor's padding (patches at position (-1, -1), audio frames past
the mask) is left out. Each item's rows stay on the device and, as BF16 host rows, in the cache the
connector saves from, until vLLM frees the hash. The reference's encoder-only instance:
integrations/furiosa-opt-vllm/furiosa_opt_vllm/multimodal.py.
"""

from __future__ import annotations


class Media:
    """A loaded media encoder, its device, and the rows of every item hash vLLM has not freed."""

    def __init__(self, engine, encoder, device):
        self.engine, self.encoder, self.device = engine, encoder, device
        self.rows: dict = {}  # hash -> device rows
        self.host: dict = {}  # hash -> BF16 host rows (the connector's encoder cache)
        self.features: dict[str, list] = {}  # request -> its media features (vLLM's mm_features)

    def _upload(self, rows):
        import torch

        return self.engine.HostTensor.from_dlpack(rows.detach().to(torch.bfloat16).contiguous()).to_hbm(self.device)

    def _image(self, pixels, positions):
        """Patches of one image (or of a video's frames, flattened), padding left out."""
        keep = ~(positions == -1).all(dim=-1)
        return self.engine.vision_language.Image(self._upload(pixels[keep]), positions[keep].tolist())

    def embed(self, feature):
        """The rows of one media item, one per placeholder position of its prompt."""
        import torch

        if feature.data is None:
            raise ValueError(f"item {feature.identifier} has no processed inputs")
        data = feature.data.get_data() if hasattr(feature.data, "get_data") else feature.data

        def tensor(key):
            v = data[key]
            if not isinstance(v, torch.Tensor):
                raise ValueError(f"the processor's {key} is not a tensor")
            return v

        if feature.modality == "image":
            (rows,) = self.encoder.vision([self._image(tensor("pixel_values"), tensor("pixel_position_ids"))])
        elif feature.modality == "video":
            pixels = tensor("pixel_values_videos")
            positions = tensor("pixel_position_ids_videos")
            (rows,) = self.encoder.vision([self._image(pixels.reshape(-1, pixels.shape[-1]),
                                                       positions.reshape(-1, positions.shape[-1]))])
        elif feature.modality == "audio":
            frames, mask = tensor("input_features_padded"), tensor("input_features_mask").bool()
            valid = int(mask.sum())
            if not bool(mask[:valid].all()):
                raise ValueError("an audio clip's valid frames precede its padding")
            (rows,) = self.encoder.audio([self.engine.vision_language.Audio(self._upload(frames[:valid]))])
        else:
            raise NotImplementedError(f"the media encoder embeds no {feature.modality}")
        want = feature.mm_position.get_num_embeds() if hasattr(feature.mm_position, "get_num_embeds") else None
        if want is not None and int(rows.shape[0]) != int(want):
            raise ValueError(f"{feature.modality} item has {rows.shape[0]} rows for {want} placeholders")
        return rows

    def update(self, so) -> None:
        """Records the media features of new requests and forgets finished ones."""
        for rid in so.finished_req_ids:
            self.features.pop(rid, None)
        for nr in so.scheduled_new_reqs:
            self.features[nr.req_id] = list(getattr(nr, "mm_features", None) or [])

    def step(self, so, save=None) -> list[str]:
        """Embeds the step's scheduled items (each hash once) and saves each through `save(cache,
        hash)`; returns the hashes embedded in this step."""
        import numpy as np
        import torch

        self.update(so)
        for h in so.free_encoder_mm_hashes:
            self.rows.pop(h, None)
            self.host.pop(h, None)
        done = []
        for rid, indices in so.scheduled_encoder_inputs.items():
            for i in indices:
                feature = self.features[rid][i]
                h = feature.identifier
                if h in self.rows:
                    continue
                rows = self.embed(feature)
                self.rows[h] = rows
                host = np.asarray(rows.to_host().numpy())
                self.host[h] = torch.from_numpy(host.astype(np.float32)).to(torch.bfloat16)
                if save is not None:
                    save(self.host, h)
                done.append(h)
        return done


def execute(media: Media, so):
    """vLLM's encoder-only step on the engine: embed and save through the EC connector (when one is
    configured), then vLLM's empty encoder output."""
    from vllm.v1.outputs import make_empty_encoder_model_runner_output
    from vllm.v1.worker.ec_connector_model_runner_mixin import ECConnectorModelRunnerMixin as Mixin

    with Mixin.maybe_get_ec_connector_output(so, encoder_cache=media.host):
        media.step(so, save=Mixin.maybe_save_ec_to_connector)
        return make_empty_encoder_model_runner_output(so)


def encoder_only(model_config) -> bool:
    """Whether vLLM runs this instance as a media encoder alone (`mm_encoder_only`)."""
    mm = getattr(model_config, "multimodal_config", None)
    return bool(getattr(mm, "mm_encoder_only", False))
