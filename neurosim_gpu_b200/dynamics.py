"""Per-neuron parameters of the soma / dendrite / adaptation tick.

Mirrors the reference parameter types so a caller's model objects carry over:
``Dynamics`` (src/neurosim_gpu/dynamics.py:8-61) holds the soma ``alpha`` and
``gain``; ``DendriticDynamics`` (src/neurosim_gpu/compartmental.py:67-183) adds
the dendrite / adaptation retention factors, the coupling and the adaptation
strength, with the same validation and the same ``from_time_constants``
(retention = exp(-dt / tau)).

The ``advance`` methods are the differentiable PyTorch form of the tick.  The
native runtimes use them only for requests that need autograd, which the CUDA
kernels do not provide (the reference does the same,
native_compartmental.py:104-108).  The inference tick always runs in CUDA.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class Dynamics:
    """Soma parameters: s' = clamp(alpha*s + (1-alpha)*gain*tanh(current + drive), 0, 1)."""

    alpha: torch.Tensor
    gain: torch.Tensor

    def __post_init__(self) -> None:
        if self.alpha.ndim != 1 or self.gain.ndim != 1:
            raise ValueError("alpha and gain must be rank-1 tensors")
        if self.alpha.shape != self.gain.shape:
            raise ValueError("alpha and gain must have the same shape")
        if torch.any((self.alpha < 0) | (self.alpha >= 1)):
            raise ValueError("alpha must satisfy 0 <= alpha < 1")
        if torch.any(self.gain < 0):
            raise ValueError("gain must be non-negative")

    @property
    def n_neurons(self) -> int:
        return self.alpha.numel()

    @property
    def beta(self) -> torch.Tensor:
        return 1.0 - self.alpha

    def advance(self, state: torch.Tensor, synaptic_current: torch.Tensor,
                drive: torch.Tensor | float = 0.0) -> torch.Tensor:
        equilibrium = self.gain * torch.tanh(synaptic_current + drive)
        return torch.clamp(self.alpha * state + self.beta * equilibrium, min=0.0, max=1.0)


@dataclass(frozen=True)
class DendriticDynamics:
    """One signed dendritic compartment and a slow negative-feedback trace."""

    soma: Dynamics
    dendrite_decay: torch.Tensor
    adaptation_decay: torch.Tensor
    coupling: torch.Tensor
    adaptation_strength: torch.Tensor

    def __post_init__(self) -> None:
        reference = self.soma.alpha
        for name, value in (
            ("soma.alpha", reference), ("soma.gain", self.soma.gain),
            ("dendrite_decay", self.dendrite_decay),
            ("adaptation_decay", self.adaptation_decay),
            ("coupling", self.coupling),
            ("adaptation_strength", self.adaptation_strength),
        ):
            if value.shape != reference.shape or value.ndim != 1:
                raise ValueError(f"{name} must have one value per neuron")
            if not value.is_floating_point():
                raise ValueError(f"{name} must be floating point")
            if value.device != reference.device or value.dtype != reference.dtype:
                raise ValueError(f"{name} must match soma device and dtype")
            if not bool(torch.isfinite(value).all()):
                raise ValueError(f"{name} must be finite")
        for name in ("dendrite_decay", "adaptation_decay"):
            value = getattr(self, name)
            if bool(((value < 0) | (value >= 1)).any()):
                raise ValueError(f"{name} must be in [0, 1)")
        if bool(((self.coupling < 0) | (self.coupling > 1)).any()):
            raise ValueError("coupling must be in [0, 1]")
        if bool((self.adaptation_strength < 0).any()):
            raise ValueError("adaptation_strength must be non-negative")

    @classmethod
    def from_time_constants(cls, soma: Dynamics, *, dt: float,
                            tau_dendrite: torch.Tensor | float,
                            tau_adaptation: torch.Tensor | float,
                            coupling: torch.Tensor | float = 0.5,
                            adaptation_strength: torch.Tensor | float = 0.2
                            ) -> "DendriticDynamics":
        """Retention factors exp(-dt/tau); scalars broadcast to one value per neuron."""
        if not math.isfinite(dt) or dt <= 0:
            raise ValueError("dt must be finite and positive")

        def vector(value, name: str) -> torch.Tensor:
            result = torch.as_tensor(value, dtype=soma.alpha.dtype, device=soma.alpha.device)
            if result.ndim == 0:
                result = result.expand_as(soma.alpha)
            if result.shape != soma.alpha.shape:
                raise ValueError(f"{name} must be scalar or have one value per neuron")
            return result

        def decay(value, name: str) -> torch.Tensor:
            tau = vector(value, name)
            if not bool((torch.isfinite(tau) & (tau > 0)).all()):
                raise ValueError(f"{name} must be finite and positive")
            return torch.exp(-dt / tau)

        return cls(soma, decay(tau_dendrite, "tau_dendrite"),
                   decay(tau_adaptation, "tau_adaptation"),
                   vector(coupling, "coupling"),
                   vector(adaptation_strength, "adaptation_strength"))

    def parameters(self) -> list[torch.Tensor]:
        """The six per-neuron vectors in kernel order."""
        return [self.soma.alpha, self.soma.gain, self.dendrite_decay, self.adaptation_decay,
                self.coupling, self.adaptation_strength]

    def advance(self, state: torch.Tensor, dendritic_state: torch.Tensor,
                adaptation_state: torch.Tensor, synaptic_current: torch.Tensor,
                drive: torch.Tensor | float = 0.0, *,
                dendritic_drive: torch.Tensor | float = 0.0
                ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """Differentiable tick: reads s_t, d_t, a_t and returns (s_t+1, d_t+1, a_t+1)."""
        dendrite = (self.dendrite_decay * dendritic_state
                    + (1.0 - self.dendrite_decay) * torch.tanh(synaptic_current + dendritic_drive))
        current = ((1.0 - self.coupling) * synaptic_current + self.coupling * dendrite
                   - self.adaptation_strength * adaptation_state)
        state = self.soma.advance(state, current, drive)
        adaptation = (self.adaptation_decay * adaptation_state
                      + (1.0 - self.adaptation_decay) * state)
        return state, dendrite, adaptation
