"""``model.triton_kernels`` configuration keys, kept as the reference defines them.

Mirrors ``TritonKernelsConfig`` (src/picotron/config/config.py:72-92): six strict boolean
opt-ins, all False by default. ``rmsnorm``, ``swiglu``, ``rope`` and ``cross_entropy``
select the sm_100a kernels of this package (``cross_entropy`` and ``adamw`` through
``kernels.CrossEntropyWithFallback(use_triton=...)`` and
``kernels.AdamWStepWithFallback(use_triton=...)``, as the reference's training loop builds
them, train_loop.py:95-100); ``attention`` is accepted for config compatibility and selects
nothing here. ``module_kwargs`` maps the switches onto the
module constructor keywords (``use_triton_rmsnorm`` and friends) that the reference's
decoder passes (picotron_decoder.py:78-101, nn/attention.py).
"""

from __future__ import annotations

from collections.abc import Mapping
from dataclasses import dataclass, fields


class ConfigValidationError(ValueError):
    """Raised when a kernel configuration is invalid (reference config.py:19-20)."""


_FIELDS = ("rmsnorm", "swiglu", "rope", "attention", "cross_entropy", "adamw")


@dataclass(frozen=True, slots=True)
class TritonKernelsConfig:
    """Explicit opt-ins for the accelerated kernels."""

    rmsnorm: bool = False
    swiglu: bool = False
    rope: bool = False
    attention: bool = False
    cross_entropy: bool = False
    adamw: bool = False

    def __post_init__(self) -> None:
        for name in _FIELDS:
            value = getattr(self, name)
            if not isinstance(value, bool):
                raise ConfigValidationError(f"'{name}' must be a boolean; got {value!r}.")

    @classmethod
    def from_mapping(cls, values: Mapping[str, object], path: str = "model.triton_kernels"):
        """Build from a mapping; unknown keys are errors, as in the reference loader."""

        if not isinstance(values, Mapping):
            raise ConfigValidationError(f"'{path}' must be a mapping.")
        known = {f.name for f in fields(cls)}
        unknown = sorted(set(values) - known)
        if unknown:
            raise ConfigValidationError(f"Unknown key(s) in '{path}': {', '.join(unknown)}.")
        return cls(**values)

    def module_kwargs(self) -> dict[str, bool]:
        """Constructor keywords of the modules this package provides."""

        return {
            "use_triton_rmsnorm": self.rmsnorm,
            "use_triton_swiglu": self.swiglu,
            "use_triton_rope": self.rope,
        }
