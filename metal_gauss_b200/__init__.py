"""metal_gauss_b200: the metal-gauss training hot path on NVIDIA B200 (sm_100a).

Drop-in surface (same names and semantics as the reference's modules):
  render / BACKENDS          metal_gauss.api
  cuda_backend.render        metal_gauss.metal_backend.render
  ext                        the reference bridge's kernel functions
  FusedAdam, SelectiveAdam   metal_gauss.fused_adam / selective_adam
  ssim, gaussian_kernel      train.ssim / train._gaussian_kernel
Batched multi-view training (one process per GPU, NCCL gradient exchange):
  engine.Trainer, engine.fit
Forward-only rendering of many views (viewer / camera paths):
  renderer.Renderer
"""

from .api import BACKENDS, render

__all__ = ["render", "BACKENDS"]
