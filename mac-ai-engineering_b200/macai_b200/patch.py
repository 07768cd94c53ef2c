"""Install the B200 gated delta rule into transformers' Qwen3.5-family models, so existing training and inference code
runs it without changes. Mirrors the reference's src/macai/patch.py (install :33-56, uninstall :77-89, installed
:92-98) for the rule swap; the reference's layer, training and LoRA patches are not part of this package.

transformers 5.x binds the rule in two ways, and both are covered:
- the module-level function `torch_chunk_gated_delta_rule` (the reference swaps this name, patch.py:27-46);
- `Qwen3_5GatedDeltaNet.__init__` stores `self.chunk_gated_delta_rule = chunk_gated_delta_rule or
  torch_chunk_gated_delta_rule`, where the first name is flash-linear-attention's kernel when fla is importable. The
  module-level `chunk_gated_delta_rule` is swapped as well, so layers built after install() bind this rule; layers
  built before it are rebound by install(model=...).

    import macai_b200.patch
    macai_b200.patch.install()                 # every later-built Qwen3.5 / Qwen3.5-MoE / Qwen3-Next model
    macai_b200.patch.install(model=model)      # and the layers of an already-built model
    with macai_b200.patch.installed():         # or only inside a block
        ...
"""
from __future__ import annotations

import contextlib
import importlib

from .gated_delta import chunk_gated_delta_rule

MODULES = ("transformers.models.qwen3_5.modeling_qwen3_5", "transformers.models.qwen3_5_moe.modeling_qwen3_5_moe",
           "transformers.models.qwen3_next.modeling_qwen3_next")
NAMES = ("torch_chunk_gated_delta_rule", "chunk_gated_delta_rule")
ATTR = "chunk_gated_delta_rule"       # the per-layer binding
_saved: dict = {}                     # (module path, name) -> original
_rebound: list = []                   # (layer, original bound function)


def install(model=None) -> list:
    """Swap the rule in every modeling module that has it; returns the (module, name) pairs patched. With model, also
    rebind the rule of every layer of that model that holds one."""
    done = []
    for path in MODULES:
        try:
            mod = importlib.import_module(path)
        except ImportError:
            continue
        for name in NAMES:
            if hasattr(mod, name) and getattr(mod, name) is not chunk_gated_delta_rule:
                _saved[(path, name)] = getattr(mod, name)
                setattr(mod, name, chunk_gated_delta_rule)
                done.append((path, name))
    if model is not None:
        for layer in model.modules():
            fn = getattr(layer, ATTR, None)
            if callable(fn) and fn is not chunk_gated_delta_rule and not isinstance(fn, type):
                _rebound.append((layer, fn))
                setattr(layer, ATTR, chunk_gated_delta_rule)
    return done


def uninstall() -> None:
    for (path, name), fn in list(_saved.items()):
        setattr(importlib.import_module(path), name, fn)
        del _saved[(path, name)]
    while _rebound:
        layer, fn = _rebound.pop()
        setattr(layer, ATTR, fn)


def patched() -> list:
    """The (module, name) pairs currently routed to this package's rule."""
    return sorted(_saved)


@contextlib.contextmanager
def installed(model=None):
    install(model=model)
    try:
        yield
    finally:
        uninstall()
