"""SigLIP vision tower + PaliGemma projector on the B200 kernels: the image
embedder the reference calls once per camera (``vlm.model.get_image_features``,
reflex/policies/pi05/modeling_pi05.py:141-158, :244), producing the 256 image
tokens of width 2048 that the prefix layers turn into the context K/V.

Per image: patch rows (rfx_patches) -> patch convolution as a GEMM with its
bias, added to the position embeddings (rfx_linear, residual epilogue) -> 27 x
[LayerNorm -> q|k|v projection -> per-image attention (rfx_vit_attention) ->
out projection + residual -> LayerNorm -> fc1 + GELU-tanh -> fc2 + residual]
-> post LayerNorm -> projector.  All images of a call are one batch of
B * 256 token rows; the launches of one batch size are captured in one CUDA
graph.  Weights are bf16 with fp32 LayerNorm parameters and biases; the MLP
width (4304) is zero-padded to 4352 and the patch length (588) to 640 so every
GEMM dimension meets the kernels' tiles (padded rows and columns contribute
exact zeros).
"""
from __future__ import annotations

import torch

from . import _lib as L
from . import kernels as K
from .config import VisionConfig


def _up(x: int, m: int) -> int:
    return (x + m - 1) // m * m


class VisionTower:
    """``get_image_features(pixels)``: [B, 3, 224, 224] fp32 images in [-1, 1]
    -> [B, 256, proj_dim] bf16 image tokens, for B up to ``max_images``."""

    def __init__(self, cfg: VisionConfig, weights: dict[str, torch.Tensor], *, max_images: int = 3,
                 device="cuda", graph: bool = True):
        self.cfg, self.dev, self.graph = cfg, torch.device(device), graph
        self.max_images = max_images
        W, F, N = cfg.width, cfg.mlp_dim, cfg.tokens
        self.Fp, self.Kp = _up(F, 128), _up(cfg.patch_dim, 64)
        dev = self.dev
        bf = dict(dtype=torch.bfloat16, device=dev)
        f32 = dict(dtype=torch.float32, device=dev)
        pre = "vision_model."

        def wb(name):
            return weights[name].to(**bf).contiguous()

        def v32(name):
            return weights[name].to(**f32).contiguous()

        pw = weights[pre + "embeddings.patch_embedding.weight"].reshape(W, -1)
        self.w_patch = torch.zeros(W, self.Kp, **bf)
        self.w_patch[:, : cfg.patch_dim] = pw.to(**bf)
        self.b_patch = v32(pre + "embeddings.patch_embedding.bias")
        self.pos = wb(pre + "embeddings.position_embedding.weight")  # [N, W]
        self.layers = []
        for l in range(cfg.num_layers):
            p = f"{pre}encoder.layers.{l}."
            a = p + "self_attn."
            w1 = torch.zeros(self.Fp, W, **bf)
            w1[:F] = wb(p + "mlp.fc1.weight")
            b1 = torch.zeros(self.Fp, **f32)
            b1[:F] = v32(p + "mlp.fc1.bias")
            w2 = torch.zeros(W, self.Fp, **bf)
            w2[:, :F] = wb(p + "mlp.fc2.weight")
            self.layers.append(dict(
                ln1_w=v32(p + "layer_norm1.weight"), ln1_b=v32(p + "layer_norm1.bias"),
                w_qkv=torch.cat([wb(a + "q_proj.weight"), wb(a + "k_proj.weight"), wb(a + "v_proj.weight")]).contiguous(),
                b_qkv=torch.cat([v32(a + "q_proj.bias"), v32(a + "k_proj.bias"), v32(a + "v_proj.bias")]).contiguous(),
                w_o=wb(a + "out_proj.weight"), b_o=v32(a + "out_proj.bias"),
                ln2_w=v32(p + "layer_norm2.weight"), ln2_b=v32(p + "layer_norm2.bias"),
                w1=w1, b1=b1, w2=w2, b2=v32(p + "mlp.fc2.bias"),
            ))
        self.post_w, self.post_b = v32(pre + "post_layernorm.weight"), v32(pre + "post_layernorm.bias")
        self.w_proj, self.b_proj = wb("projector.linear.weight"), v32("projector.linear.bias")
        # activations for max_images images
        T = max_images * N
        self.img = torch.zeros(max_images, cfg.channels, cfg.image, cfg.image, **f32)
        self.patch_rows = torch.zeros(T, self.Kp, **bf)
        self.pos_rep = self.pos.repeat(max_images, 1).contiguous()
        self.x = torch.zeros(T, W, **bf)       # residual stream
        self.h = torch.zeros(T, W, **bf)       # LayerNorm output
        self.qkv = torch.zeros(T, 3 * W, **bf)
        self.attn = torch.zeros(T, W, **bf)
        self.f = torch.zeros(T, self.Fp, **bf)
        self.out = torch.zeros(T, cfg.proj_dim, **bf)
        self.split_ws = None
        self._plans: dict[int, K.Plan] = {}

    # ------------------------------------------------------------------ ops
    def ops(self, B: int) -> list:
        """The launch list for B images (descriptors in order)."""
        cfg, N = self.cfg, self.cfg.tokens
        T = B * N
        ops = [
            K.copy_rows_desc(dst=self.x, src=self.pos_rep, rows=T, width=cfg.width, dst_rows_per_group=T, group=T),
            K.patches_desc(image=self.img[:B], out=self.patch_rows, patch=cfg.patch),
            K.linear_desc(w=self.w_patch, x=self.patch_rows, T=T, S=T, epilogue=L.RFX_EPI_RESIDUAL, y=self.x,
                          bias=self.b_patch),
        ]
        scale = cfg.head_dim ** -0.5
        for ly in self.layers:
            ops += [
                K.layer_norm_desc(x=self.x, y=self.h, w=ly["ln1_w"], b=ly["ln1_b"], eps=cfg.eps, T=T),
                K.linear_desc(w=ly["w_qkv"], x=self.h, T=T, S=T, y=self.qkv, bias=ly["b_qkv"]),
                K.vit_attention_desc(qkv=self.qkv, out=self.attn, B=B, N=N, H=cfg.num_heads, D=cfg.head_dim,
                                     scale=scale),
                K.linear_desc(w=ly["w_o"], x=self.attn, T=T, S=T, epilogue=L.RFX_EPI_RESIDUAL, y=self.x,
                              bias=ly["b_o"]),
                K.layer_norm_desc(x=self.x, y=self.h, w=ly["ln2_w"], b=ly["ln2_b"], eps=cfg.eps, T=T),
                K.linear_desc(w=ly["w1"], x=self.h, T=T, S=T, epilogue=L.RFX_EPI_GELU, y=self.f, bias=ly["b1"]),
                K.linear_desc(w=ly["w2"], x=self.f, T=T, S=T, epilogue=L.RFX_EPI_RESIDUAL, y=self.x, bias=ly["b2"]),
            ]
        ops += [
            K.layer_norm_desc(x=self.x, y=self.h, w=self.post_w, b=self.post_b, eps=cfg.eps, T=T),
            K.linear_desc(w=self.w_proj, x=self.h, T=T, S=T, y=self.out, bias=self.b_proj),
        ]
        lin = [d for d in ops if isinstance(d, L.LinearDesc)]
        need = max((K.linear_workspace_bytes(d) for d in lin), default=0)
        if need:
            if self.split_ws is None or self.split_ws.numel() < need + 256:
                self.split_ws = K.linear_workspace(need + 256, self.dev)
            for d in lin:
                d.workspace, d.workspace_bytes = K.aligned_ptr(self.split_ws, 256), need
        return ops

    def _plan(self, B: int) -> K.Plan:
        plan = self._plans.get(B)
        if plan is None:
            plan = K.Plan()
            for d in self.ops(B):
                plan.add(d)
            self._plans[B] = plan
        return plan

    def launch(self, B: int) -> None:
        """Runs the tower over the first B images of ``self.img`` on the current stream."""
        plan = self._plan(B)
        if self.graph:
            if not plan.captured:
                s = torch.cuda.Stream(device=self.dev)
                s.wait_stream(torch.cuda.current_stream(self.dev))
                with torch.cuda.stream(s):
                    plan.run()  # loads the kernels outside capture
                    plan.capture(s)
                torch.cuda.current_stream(self.dev).wait_stream(s)
            plan.replay()
        else:
            plan.run()

    def get_image_features(self, pixels: torch.Tensor) -> torch.Tensor:
        """[B, 3, H, W] images (host or device, any float dtype) -> [B, 256, proj_dim] bf16."""
        B = pixels.shape[0]
        if B < 1 or B > self.max_images:
            raise ValueError(f"get_image_features: 1..{self.max_images} images per call")
        if tuple(pixels.shape[1:]) != (self.cfg.channels, self.cfg.image, self.cfg.image):
            raise ValueError("get_image_features: images must be [B, %d, %d, %d]"
                             % (self.cfg.channels, self.cfg.image, self.cfg.image))
        self.img[:B].copy_(pixels, non_blocking=True)
        self.launch(B)
        return self.out[: B * self.cfg.tokens].view(B, self.cfg.tokens, self.cfg.proj_dim)

    def flops(self, B: int) -> float:
        """GEMM and attention FLOPs of one call over B images (unpadded shapes)."""
        c = self.cfg
        T, W, F = B * c.tokens, c.width, c.mlp_dim
        per_layer = 2 * T * W * (3 * W + W + 2 * F) + 4 * B * c.num_heads * c.tokens * c.tokens * c.head_dim
        return float(2 * T * W * c.patch_dim + c.num_layers * per_layer + 2 * T * W * c.proj_dim)

    def weight_bytes(self) -> int:
        n = self.w_patch.numel() + self.w_proj.numel()
        for ly in self.layers:
            n += ly["w_qkv"].numel() + ly["w_o"].numel() + ly["w1"].numel() + ly["w2"].numel()
        return 2 * n


def image_features(cfg: VisionConfig, weights, pixels: torch.Tensor, **kw) -> torch.Tensor:
    """One-shot helper: builds a tower for ``pixels.shape[0]`` images and runs it."""
    tower = VisionTower(cfg, weights, max_images=pixels.shape[0], **kw)
    return tower.get_image_features(pixels)

