"""Policy-level entry points with the reference's call signatures, over the
rfx engines (the denoising half of Reflex's PI0.5 / PI0 policies).

* ``PI05Model.denoise_step(prefix_pad_masks, prefix_att_masks, state, x_t,
  timestep)`` -> v_t: reflex/policies/pi05/modeling_pi05.py:1181-1241.
* ``PI05Model.sample_actions(images, img_masks, tokens, masks, state,
  noise=None, num_steps=None, incremental_input=False)`` -> actions:
  modeling_pi05.py:1244-1425 (streaming branch :1282-1357).
* ``PI05Policy.predict_action_chunk(batch, noise=None, num_steps=None,
  incremental_input=False)`` / ``select_action(batch, noise=None)`` /
  ``reset()``: modeling_pi05.py:1640-1700.
* ``PI0Model`` / ``PI0Policy``: the same for reflex/policies/pi0/
  modeling_pi0.py:740-845, 1001-1040 (``sample_actions`` and
  ``predict_action_chunk`` without ``incremental_input``).

What enters where the reference starts from raw observations: ``images``
are either the cameras' images (a list of [B, 3, 224, 224] tensors, one per
camera, or one [B, n_cams, 3, 224, 224] tensor), which a model built with a
``vision`` tower (reflex_b200.vision.VisionTower, the SigLIP tower and
projector of ``get_image_features``, modeling_pi05.py:141-158,244) turns into
image tokens, or the image tokens themselves [B, frame_len, vlm_width] (one
frame: every camera's 256 tokens, cameras in order).  The language embedding
table is not part of this library: ``tokens`` are the instruction's token
embeddings [B, n_lang, vlm_width].
With prefix-layer weights the model runs them through the prefix layers
into the KV rings (PrefixEngine: the instruction once, each frame into the
sliding window, the oldest frame evicted); without them the caller fills the
rings (``load_prefix_cache``) and passes ``images=None, tokens=None``.
Input normalization and output unnormalization by dataset statistics
(normalize_inputs / unnormalize_outputs) are identities here.
"""
from __future__ import annotations

import dataclasses
from collections import deque

import torch

from .config import ExpertConfig
from .expert import ActionExpertEngine
from .prefix import PrefixEngine


class PI05Model:
    """The denoising part of PI05Model on the rfx engines.

    Ring layout per layer: slots [0, n_lang) hold the instruction, then
    ``window_frames`` frame slots of ``frame_len`` (frame f in slot
    f % window_frames).  ``fused`` selects the persistent chunk executor
    (at most 64 suffix tokens per GPU; the default where they fit) over one
    launch per op."""

    variant = "pi05"

    def __init__(self, cfg: ExpertConfig, weights: dict, *, prefix_cfg: ExpertConfig | None = None,
                 prefix_weights: dict | None = None, batch: int = 1, n_lang: int = 0, frame_len: int = 0,
                 window_frames: int = 2, capacity: int | None = None, device="cuda", fused: bool | None = None,
                 vision=None):
        if cfg.variant != self.variant:
            raise ValueError(f"{type(self).__name__} needs a {self.variant} config")
        cap = capacity or max(1, n_lang + window_frames * frame_len)
        if cap < n_lang + window_frames * frame_len:
            raise ValueError(f"capacity {cap} < instruction {n_lang} + {window_frames} frames of {frame_len}")
        if fused is None:
            fused = batch * cfg.suffix_len <= 64
        self.cfg, self.B, self.dev = cfg, batch, torch.device(device)
        self.n_lang, self.frame_len, self.window_frames = n_lang, frame_len, window_frames
        self.num_inference_steps = cfg.num_steps
        self.engine = ActionExpertEngine(cfg, weights, batch=batch, capacity=cap, n_ctx=0, device=device,
                                         scale_dtype=torch.float32, fused=fused)
        self._step_engine = None
        self.instruction = self.frames = None
        if prefix_weights is not None:
            if prefix_cfg is None or n_lang < 1 or frame_len < 1:
                raise ValueError("prefix_weights need prefix_cfg, n_lang >= 1 and frame_len >= 1")
            self.instruction = PrefixEngine(prefix_cfg, prefix_weights, self.engine.rings, pinned=0,
                                            frame_len=n_lang, window_frames=1, batch=batch, device=device)
            self.frames = PrefixEngine(prefix_cfg, self.instruction, self.engine.rings, pinned=n_lang,
                                       frame_len=frame_len, window_frames=window_frames, batch=batch, device=device)
        self.frames_seen = 0
        self.has_instruction = False
        self.vision = vision

    # ------------------------------------------------------------ prefix ---
    @property
    def prefix_length(self) -> int:
        """Valid prefix tokens in the rings (instruction + frames in the window)."""
        return self.n_lang * self.has_instruction + min(self.frames_seen, self.window_frames) * self.frame_len

    def load_prefix_cache(self, layer: int, k: torch.Tensor, v: torch.Tensor, slot_base: int = 0) -> None:
        """Puts prefix K/V [B, 1, L, 256] computed elsewhere (post-RoPE) into
        slots [slot_base, slot_base + L) of one layer's ring (quantized)."""
        self.engine.load_context(layer, k, v, region_base=0, region_off=slot_base, region_len=self.engine.capacity)

    def set_prefix(self, n_tokens: int, instruction: bool = True, frames: int = 0) -> None:
        """Declares what the rings hold after load_prefix_cache: the
        instruction (if any) and `frames` frames; n_tokens must match."""
        self.has_instruction, self.frames_seen = instruction, frames
        if n_tokens != self.prefix_length:
            raise ValueError(f"{n_tokens} prefix tokens, the layout gives {self.prefix_length}")

    def embed_images(self, images):
        """Camera images -> image tokens [B, n_cams * 256, proj_dim] through the
        vision tower (cameras batched into one call, in camera order as the
        reference concatenates them, modeling_pi05.py:236-253); image tokens
        pass through unchanged."""
        if images is None:
            return None
        if isinstance(images, (list, tuple)):
            images = torch.stack([torch.as_tensor(im) for im in images], 1)
        if images.dim() != 5:
            return images
        if self.vision is None:
            raise ValueError("camera images given but the model has no vision tower")
        B, nc = images.shape[:2]
        feats = self.vision.get_image_features(images.reshape(B * nc, *images.shape[2:]))
        return feats.reshape(B, nc * feats.shape[1], feats.shape[2])

    def _prefill(self, images, tokens, incremental_input: bool) -> None:
        images = self.embed_images(images)
        if tokens is not None and (not incremental_input or not self.has_instruction):
            if self.instruction is None:
                raise ValueError("instruction embeddings given but the model has no prefix-layer weights")
            self.instruction.run(tokens.reshape(self.B * self.n_lang, -1))
            self.has_instruction = True
            self.frames_seen = 0
            self.frames.frames = 0
        elif not incremental_input and images is not None:
            self.frames_seen = 0  # a full (non-incremental) observation restarts the window
            if self.frames is not None:
                self.frames.frames = 0
        if images is not None:
            if self.frames is None:
                raise ValueError("image embeddings given but the model has no prefix-layer weights")
            self.frames.run(images.reshape(self.B * self.frame_len, -1))
            self.frames_seen += 1

    @staticmethod
    def _check_masks(*masks) -> None:
        for m in masks:
            if m is not None and not bool(torch.as_tensor(m).bool().all()):
                raise ValueError("padded prefix tokens are not supported by sample_actions "
                                 "(denoise_step takes a prefix padding mask)")

    # ------------------------------------------------------------- steps ---
    def _step(self) -> ActionExpertEngine:
        """A one-step engine over the same weights and rings: x_new = x_t +
        bf16(1.0 * v_t), so v_t = x_new - x_t (exact for the bf16 velocity)."""
        eng = self.engine
        if self._step_engine is None or self._step_engine.n_ctx != eng.n_ctx:
            cfg1 = dataclasses.replace(self.cfg, num_steps=1)
            self._step_engine = ActionExpertEngine(cfg1, eng, batch=self.B, capacity=eng.capacity, n_ctx=eng.n_ctx,
                                                   device=self.dev, scale_dtype=torch.float32, fused=False,
                                                   timesteps=[1.0], dt=1.0)
        return self._step_engine

    def _context(self, n_ctx: int) -> None:
        eng = self.engine
        if n_ctx != eng.n_ctx:
            eng.set_context_length(n_ctx)  # the window is still filling: new launch plan
        eng.set_context_mask(None)

    @torch.no_grad()
    def denoise_step(self, prefix_pad_masks: torch.Tensor, prefix_att_masks: torch.Tensor, state: torch.Tensor,
                     x_t: torch.Tensor, timestep: torch.Tensor) -> torch.Tensor:
        """One denoising step over the cached prefix -> v_t [B, chunk, action_dim]
        (fp32 holding the bf16 velocity).  The suffix rows see every
        unpadded prefix token whatever the prefix's own attention pattern
        (cumsum order, reflex/policies/pi05/utils.py:210-215), so
        prefix_att_masks only has to have the prefix's length; all streams
        share one timestep."""
        B, Lc = prefix_pad_masks.shape
        if B != self.B or prefix_att_masks.shape[-1] != Lc:
            raise ValueError(f"prefix masks must be [{self.B}, {Lc}]")
        ts = torch.as_tensor(timestep, dtype=torch.float32).reshape(-1)
        if not bool((ts == ts[0]).all()):
            raise ValueError("denoise_step: every stream of the batch takes the same timestep")
        if Lc != self.engine.n_ctx:
            self.engine.set_context_length(Lc)
        step = self._step()
        pad = prefix_pad_masks.to(self.dev).bool()
        # padded slots are invisible and the suffix positions continue after
        # each stream's unpadded prefix tokens (set_context_mask)
        step.set_context_mask(None if bool(pad.all()) else pad)
        step.t.fill_(float(ts[0]))
        x_t = x_t.to(self.dev, torch.float32)
        step.set_inputs(x_t, state if self.cfg.variant == "pi0" else None)
        step.launch_chunk()
        return (step.x - x_t).to(torch.bfloat16).float()

    @torch.no_grad()
    def sample_actions(self, images, img_masks, tokens, masks, state, noise=None, num_steps=None,
                       incremental_input: bool = False) -> torch.Tensor:
        """Prefill (instruction and/or new frame, if given), then the Euler loop
        of num_steps denoising steps from noise -> actions [B, chunk, action_dim]."""
        if num_steps is not None and num_steps != self.cfg.num_steps:
            raise ValueError(f"the engine is built for {self.cfg.num_steps} steps, got {num_steps}")
        self._check_masks(img_masks, masks)
        self._prefill(images, tokens, incremental_input)
        self._context(self.prefix_length)
        if noise is None:
            noise = torch.randn(self.B, self.cfg.chunk_size, self.cfg.action_dim, device=self.dev)
        eng = self.engine
        eng.set_inputs(noise.to(self.dev, torch.float32), state if self.cfg.variant == "pi0" else None)
        eng.launch_chunk()
        return eng.x.clone()


class PI0Model(PI05Model):
    """PI0: state token + action/time MLP suffix, plain RMSNorm."""

    variant = "pi0"

    @torch.no_grad()
    def sample_actions(self, images, img_masks, tokens, masks, state, noise=None, num_steps=None) -> torch.Tensor:
        """reflex/policies/pi0/modeling_pi0.py:785: prefill, then the Euler loop."""
        if state is None:
            raise ValueError("PI0 needs the robot state")
        return super().sample_actions(images, img_masks, tokens, masks, state, noise, num_steps,
                                      incremental_input=images is not None and tokens is None)


class PI05Policy:
    """Inference wrapper of PI05Model with the reference's batch interface.
    Batch keys: "observation.state" [B, state_dim], and (when the model has
    prefix-layer weights) "observation.image_embeddings" [B, frame_len, W]
    and "observation.language_embeddings" [B, n_lang, W]."""

    def __init__(self, model: PI05Model, n_action_steps: int | None = None, action_dim: int | None = None):
        self.model = model
        self.n_action_steps = n_action_steps or model.cfg.chunk_size
        if self.n_action_steps > model.cfg.chunk_size:
            raise ValueError(f"n_action_steps ({self.n_action_steps}) cannot be greater than chunk_size "
                             f"({model.cfg.chunk_size})")
        self.action_dim = action_dim or model.cfg.action_dim
        self.reset()

    def reset(self) -> None:
        """Clears the action queue (call when the environment resets)."""
        self._action_queue = deque([], maxlen=self.n_action_steps)

    def _inputs(self, batch: dict):
        return (batch.get("observation.image_embeddings"), batch.get("observation.language_embeddings"),
                batch.get("observation.state"))

    @torch.no_grad()
    def predict_action_chunk(self, batch: dict, noise: torch.Tensor | None = None, num_steps: int | None = None,
                             incremental_input: bool = False) -> torch.Tensor:
        """Action chunk [B, n_action_steps, action_dim] (modeling_pi05.py:1649)."""
        images, tokens, state = self._inputs(batch)
        actions = self.model.sample_actions(images, None, tokens, None, state, noise=noise, num_steps=num_steps,
                                            incremental_input=incremental_input)
        return actions[:, :self.n_action_steps, :self.action_dim]

    @torch.no_grad()
    def select_action(self, batch: dict, noise: torch.Tensor | None = None) -> torch.Tensor:
        """One action [B, action_dim] from the queue, refilled with a new chunk
        when empty (modeling_pi05.py:1681)."""
        if len(self._action_queue) == 0:
            actions = self.predict_action_chunk(batch, noise=noise)
            self._action_queue.extend(actions.transpose(0, 1)[: self.n_action_steps])
        return self._action_queue.popleft()


class PI0Policy(PI05Policy):
    @torch.no_grad()
    def predict_action_chunk(self, batch: dict, noise: torch.Tensor | None = None) -> torch.Tensor:
        """reflex/policies/pi0/modeling_pi0.py:1010."""
        images, tokens, state = self._inputs(batch)
        actions = self.model.sample_actions(images, None, tokens, None, state, noise=noise)
        return actions[:, :self.n_action_steps, :self.action_dim]
