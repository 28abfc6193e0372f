"""Single render interface with swappable backends (metal_gauss/api.py:1-27).

`cuda` is this package's sm_100a backend. `torch_ref` delegates to the
reference package's pure-PyTorch renderer when it is installed (it is the
correctness oracle there); `metal` needs an Apple GPU and is refused here.
Asking for a backend either uses it or raises: nothing is silently substituted.
"""

from __future__ import annotations

BACKENDS = ("torch_ref", "cuda")


def render(*args, backend: str = "cuda", **kwargs):
    if backend == "cuda":
        from . import cuda_backend
        return cuda_backend.render(*args, **kwargs)
    if backend == "torch_ref":
        try:
            from metal_gauss import torch_ref  # the reference package, if installed
        except ImportError as e:
            raise RuntimeError(
                "torch_ref backend needs the metal_gauss package (the reference) on the path. "
                "Refusing to silently substitute a different renderer.") from e
        return torch_ref.render(*args, **kwargs)
    if backend == "metal":
        raise RuntimeError("metal backend requires an Apple GPU; use backend='cuda'. "
                           "Refusing to silently substitute a different renderer.")
    raise ValueError(f"unknown backend {backend!r}; expected one of {BACKENDS}")
