"""Module-name alias so ``from <pkg>.triton_impl import DDPM`` works as a drop-in
for the reference's ``from triton_impl import DDPM`` (no Triton is involved)."""

from .ddpm import DDPM, _check_inputs

__all__ = ["DDPM", "_check_inputs"]
