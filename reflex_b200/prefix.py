"""Streaming frame update of the prefix (VLM) layers on the rfx kernels.

Each new frame of ``frame_len`` patch embeddings runs through the prefix
layers (Gemma-2B shapes): input norm -> QKV + RoPE -> attention of the frame
over the cached context (pinned instruction prefix + the newest window frame;
the frame being evicted is masked out) and over itself (bidirectional) ->
o_proj + residual -> post-attention norm -> gate/up + GeGLU -> down_proj +
residual; then the frame's post-RoPE K/V are quantize-appended into the
layer's ring in the evicted frame's slots.  This is the streaming path of
reflex/policies/pi05/modeling_pi05.py:1282-1333 (evict the oldest frame, then
prefill the new one, streaming_attention.py:281-470) with the prefix attention
of the non-streaming path (:1379-1401), and the rings are the ones the action
expert reads.

Ring layout per layer: slots [0, pinned) hold the instruction prefix, then
``window_frames`` frame slots of ``frame_len`` each; frame f goes to slot
f % window_frames.  Positions of a new frame continue after the context it
attends to (pinned + the other window frames), as the reference's streaming
prefill counts them (modeling_pi05.py:1301-1316).
"""
from __future__ import annotations

import torch

from . import _lib as L
from . import kernels as K
from .config import ExpertConfig
from .expert import fused_gate_up_weight, fused_qkv_weight
from .synthetic import rope_table


class PrefixEngine:
    """``weights`` is a state dict of the prefix layers (separate or fused
    projections) or another PrefixEngine whose packed weights are shared
    (e.g. one engine for the pinned instruction, pinned=0 and
    window_frames=1, and one for the observation frames over the same rings).
    ``ops(slot, prior)`` also serves the window while it fills: ``prior``
    frames (slots 0 .. prior-1) are in the window before the new one."""

    def __init__(self, cfg: ExpertConfig, weights, rings: list, *, pinned: int, frame_len: int,
                 window_frames: int = 2, batch: int = 1, device="cuda", kv_splits: int = 0):
        if cfg.num_kv_heads != 1 or cfg.head_dim != 256:
            raise ValueError("the kernels serve one 256-wide KV head (MQA)")
        if len(rings) != cfg.num_layers:
            raise ValueError("one ring per prefix layer")
        self.cfg, self.B, self.dev = cfg, batch, torch.device(device)
        self.pinned, self.frame_len, self.window_frames = pinned, frame_len, window_frames
        self.rings = rings
        cap = pinned + window_frames * frame_len
        if rings[0].capacity < cap:
            raise ValueError(f"rings hold {rings[0].capacity} slots, the window needs {cap}")
        self.n_ctx = cap
        dev = self.dev
        bf = lambda t: t.to(dev, torch.bfloat16).contiguous()  # noqa: E731
        Lh, W, H, D, F = cfg.num_layers, cfg.width, cfg.num_heads, cfg.head_dim, cfg.mlp_dim
        if isinstance(weights, PrefixEngine):
            src = weights
            self.w_qkv, self.w_o, self.w_gu, self.w_down = src.w_qkv, src.w_o, src.w_gu, src.w_down
            self.a_in, self.a_post = src.a_in, src.a_post
        else:
            self.w_qkv, self.w_o, self.w_gu, self.w_down, self.a_in, self.a_post = [], [], [], [], [], []
            for l in range(Lh):
                p = f"layers.{l}."
                self.w_qkv.append(K.pack_weight(L.RFX_PACK_QKV_ROPE, bf(fused_qkv_weight(weights, p))))
                self.w_o.append(bf(weights[p + "o_proj.weight"]))
                self.w_gu.append(K.pack_weight(L.RFX_PACK_GATE_UP, bf(fused_gate_up_weight(weights, p))))
                self.w_down.append(bf(weights[p + "down_proj.weight"]))
                self.a_in.append(weights[p + "input_layernorm.weight"].to(dev, torch.float32).contiguous())
                self.a_post.append(weights[p + "post_attention_layernorm.weight"].to(dev, torch.float32).contiguous())
        T = batch * frame_len
        self.T = T
        z = lambda *s, dt=torch.bfloat16: torch.zeros(*s, dtype=dt, device=dev)  # noqa: E731
        self.h = z(T, W)
        self.xn = z(T, W)
        self.q = z(batch, H, frame_len, D)
        self.k_new, self.v_new = z(T, D), z(T, D)
        self.attn_out = z(T, H * D)
        self.act = z(T, F)
        self.rope = rope_table(cfg.max_position_embeddings, D, cfg.rope_theta).to(dev)
        self._state = {}  # (slot, prior) -> (positions, context validity)
        self.kv_splits = kv_splits
        self.workspace = None
        self.split_ws = None  # split-K workspace of the GEMMs (zero-filled; one stream)
        self.frames = 0  # frames appended so far

    def load_context(self, layer: int, k: torch.Tensor, v: torch.Tensor, slot_base: int = 0) -> None:
        """Quantize-appends K/V [B, 1, L, D] at slots [slot_base, slot_base + L)."""
        K.kv_quant_append(k.to(self.dev, torch.bfloat16).contiguous(), v.to(self.dev, torch.bfloat16).contiguous(),
                          self.rings[layer], 0, slot_base, self.rings[layer].capacity)

    def set_frame(self, emb: torch.Tensor) -> None:
        """The new frame's embeddings [B, frame_len, width]."""
        self.h.copy_(emb.reshape(self.T, -1), non_blocking=True)

    def _positions_and_valid(self, slot: int, prior: int):
        """Positions of the new frame's tokens and the context it sees when it
        replaces frame slot `slot` with `prior` frames in the window: the
        pinned prefix plus the window's other filled slots (slots 0 .. prior-1
        while the window fills, every slot but `slot` once it is full).  The
        positions continue after that context, as the reference's streaming
        prefill counts them (modeling_pi05.py:1301-1316)."""
        key = (slot, prior)
        if key not in self._state:
            W, F, P = self.window_frames, self.frame_len, self.pinned
            if not 0 <= prior <= W - 1 or not 0 <= slot < W or (prior < W - 1 and slot != prior):
                raise ValueError(f"frame slot {slot} with {prior} prior frames in a window of {W}")
            pos = P + prior * F + torch.arange(F, dtype=torch.int32)
            m = torch.zeros(self.B, self.rings[0].capacity, dtype=torch.uint8)
            m[:, :P] = 1
            for s in range(W):
                if s != slot and (s < prior or prior == W - 1):
                    m[:, P + s * F: P + (s + 1) * F] = 1
            self._state[key] = (pos.repeat(self.B).to(self.dev), m.to(self.dev))
        return self._state[key]

    @property
    def positions(self):
        return self._positions_and_valid(0, self.window_frames - 1)[0]

    def ops(self, slot: int, prior: int | None = None) -> list:
        """Launch list of one frame update that replaces frame slot `slot`
        (`prior` frames already in the window; default: a full window)."""
        cfg, B, S, T = self.cfg, self.B, self.frame_len, self.T
        H, D = cfg.num_heads, cfg.head_dim
        base = self.pinned + slot * self.frame_len
        positions, valid = self._positions_and_valid(slot, self.window_frames - 1 if prior is None else prior)
        out = [("barrier", None, None)]
        attn_descs = []
        for l in range(cfg.num_layers):
            out.append(("norm", K.norm_desc(x=self.h, y=self.xn, S=S, norm_a1=self.a_in[l], eps=cfg.eps), None))
            out.append(("linear", K.linear_desc(
                w=self.w_qkv[l], x=self.xn, T=T, S=S, epilogue=L.RFX_EPI_QKV_ROPE, rope_table=self.rope,
                positions=positions, q_out=self.q, k_out=self.k_new, v_out=self.v_new, num_q_heads=H), None))
            # every one of the frame's query tiles visits every key block:
            # dequantize the context once per layer (RFX_KV_DENSE)
            ad = K.attention_desc(q=self.q, k_new=self.k_new, v_new=self.v_new, ring=self.rings[l], n_ctx=self.n_ctx,
                                  out=self.attn_out, softmax_scale=D ** -0.5, ctx_valid=valid,
                                  kv_splits=self.kv_splits, kv_source=L.RFX_KV_DENSE)
            attn_descs.append(ad)
            out.append(("attn", ad, None))
            out.append(("linear", K.linear_desc(w=self.w_o[l], x=self.attn_out, T=T, S=S,
                                                epilogue=L.RFX_EPI_RESIDUAL, y=self.h), None))
            out.append(("norm", K.norm_desc(x=self.h, y=self.xn, S=S, norm_a1=self.a_post[l], eps=cfg.eps), None))
            out.append(("linear", K.linear_desc(w=self.w_gu[l], x=self.xn, T=T, S=S, epilogue=L.RFX_EPI_GEGLU,
                                                y=self.act), None))
            out.append(("linear", K.linear_desc(w=self.w_down[l], x=self.act, T=T, S=S,
                                                epilogue=L.RFX_EPI_RESIDUAL, y=self.h), None))
            kv = self.k_new.view(B, 1, S, D)
            out.append(("quant", K.kv_quant_desc(kv, self.v_new.view(B, 1, S, D), self.rings[l], base, 0,
                                                 self.frame_len), None))
        need = max(K.attention_workspace_bytes(d) for d in attn_descs)
        if need and (self.workspace is None or self.workspace.numel() < need + 1024):
            self.workspace = torch.zeros(need + 1024, dtype=torch.uint8, device=self.dev)
        for d in attn_descs:
            if need:
                d.workspace, d.workspace_bytes = K.aligned_ptr(self.workspace, 1024), need
        lin = [d for kind, d, _ in out if kind == "linear"]
        need = max(K.linear_workspace_bytes(d) for d in lin)
        if need and (self.split_ws is None or self.split_ws.numel() < need + 256):
            self.split_ws = K.linear_workspace(need + 256, self.dev)
        for d in lin:
            if need:
                d.workspace, d.workspace_bytes = K.aligned_ptr(self.split_ws, 256), need
        return out

    def run(self, emb: torch.Tensor | None = None) -> None:
        """One frame update through the direct entry points (eager); the
        window fills first (frame f goes to slot f % window_frames)."""
        if emb is not None:
            self.set_frame(emb)
        W = self.window_frames
        for kind, desc, _ in self.ops(self.frames % W, min(self.frames, W - 1)):
            if kind != "barrier":
                K.Plan.run_direct(desc)
        self.frames += 1
