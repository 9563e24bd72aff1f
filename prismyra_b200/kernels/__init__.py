"""Kernel adapters: the plugin interface through which the B200 routed-expert layer is installed into a model.

Mirrors the reference's registry (prismyra/kernels/__init__.py:20-134) so that code written against
``prismyra.kernels`` can switch to ``prismyra_b200.kernels`` unchanged:

* an :class:`Adapter` says which architectures it handles (``supports``) and replaces modules (``replace``);
* ``replace`` returns an :class:`Applied` record of :class:`Swap` entries, each with the number of modules it
  touched and the number the configuration implies;
* :func:`apply` fails closed -- a count that differs from the expected one raises :class:`AdapterError`,
  because a swap that matched nothing is indistinguishable from one that worked -- and, with
  ``required=True``, also raises when no adapter claims the model or when any replacement was skipped.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Protocol

from torch import nn


@dataclass(frozen=True)
class Swap:
    """One replacement: its name, how many modules it replaced, and the count the configuration implies
    (``None`` when the replacement is verified some other way, which ``verified`` then describes)."""

    name: str
    replaced: int
    expected: int | None = None
    verified: str | None = None


@dataclass
class Applied:
    """The outcome of one adapter's ``replace``: swaps made, replacements skipped (with the reason) and notes on
    the limits of replacements that were made.  Holds no timings."""

    adapter: str
    swaps: list[Swap] = field(default_factory=list)
    skipped: list[str] = field(default_factory=list)
    notes: list[str] = field(default_factory=list)

    @property
    def ok(self) -> bool:
        for s in self.swaps:
            if s.expected is not None and s.replaced != s.expected:
                return False
        return True

    def summary(self) -> str:
        words = [f"{s.name}={s.replaced}" for s in self.swaps]
        if self.skipped:
            words.append("skipped=" + ",".join(self.skipped))
        return self.adapter + ": " + " ".join(words)

    def as_dict(self) -> dict:
        return {
            "adapter": self.adapter,
            "complete": self.ok and not self.skipped,
            "applied": {s.name: s.replaced for s in self.swaps},
            "verified": {s.name: s.verified for s in self.swaps if s.verified},
            "skipped": list(self.skipped),
            "notes": list(self.notes),
        }


class Adapter(Protocol):
    name: str

    def supports(self, config) -> bool:
        """True when this adapter's kernels were built for this architecture and shape."""

    def replace(self, model: nn.Module, config) -> Applied:
        """Replace every module it can (idempotently) and report what it did."""


class AdapterError(RuntimeError):
    """The model is not the one an adapter expects, or a required kernel could not be applied."""


_ADAPTERS: list[Adapter] = []


def register(adapter: Adapter) -> Adapter:
    _ADAPTERS.append(adapter)
    return adapter


def find(config) -> Adapter | None:
    return next((a for a in _ADAPTERS if a.supports(config)), None)


def apply(model: nn.Module, config, required: bool = False) -> Applied:
    """Install the kernels an adapter provides for ``config``'s architecture and return what happened."""
    adapter = find(config)
    if adapter is None:
        if required:
            raise AdapterError(
                f"no adapter for {getattr(config, 'architectures', None)}; pass required=False to run without "
                "the B200 kernels"
            )
        return Applied(adapter="none", skipped=["no adapter for this architecture"])
    applied = adapter.replace(model, config)
    if not applied.ok:
        wrong = "; ".join(
            f"{s.name} replaced {s.replaced} of an expected {s.expected}"
            for s in applied.swaps
            if s.expected is not None and s.replaced != s.expected
        )
        raise AdapterError(f"{adapter.name} found a model it does not recognise: {wrong}")
    if required and applied.skipped:
        raise AdapterError(
            f"{adapter.name} could not apply every kernel: " + "; ".join(applied.skipped)
            + " -- pass required=False to serve without it, or fix what the message names and retry"
        )
    return applied


from . import qwen3_moe as _qwen3_moe  # noqa: E402,F401  (registers its adapter)

__all__ = ["Adapter", "AdapterError", "Applied", "Swap", "apply", "find", "register"]
