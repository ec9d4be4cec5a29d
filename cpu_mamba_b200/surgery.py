"""Putting the B200 block into an existing model (src/cpu_mamba/surgery.py).

Two routes, as in the reference:

1. stub-then-import -- ``install_mamba_ssm_stub()`` makes ``from mamba_ssm
   import Mamba`` return this package's ``CPUMamba`` (the GPU block), so model
   code written against mamba_ssm builds B200 blocks directly;
2. build-then-swap -- ``swap_mamba_to_b200(model)`` walks an already-built
   model and replaces every ``mamba_ssm.Mamba`` block (and every block of the
   reference's CPU implementation, ``cpu_mamba.CPUMamba``) by this package's
   block, moving the weights over through ``state_dict`` (mamba_ssm layout on
   both sides) and onto the replaced block's device and dtype.

``swap_mamba_to_cpu`` is the reference's name for route 2 and is kept as an
alias, so code that calls it keeps working after switching packages.
"""
from __future__ import annotations

import sys
import types

import torch.nn as nn

from .module import CPUMamba


def install_mamba_ssm_stub(force: bool = False) -> None:
    """Register a ``mamba_ssm`` module whose ``Mamba`` is this package's block
    (surgery.py:29-44).  An already-imported ``mamba_ssm`` is left alone unless
    ``force``."""
    if "mamba_ssm" in sys.modules and not force:
        return
    stub = types.ModuleType("mamba_ssm")
    stub.Mamba = CPUMamba
    stub.__version__ = "cpu-mamba-b200-stub"
    sys.modules["mamba_ssm"] = stub


def _foreign_block_classes() -> tuple:
    """Block classes to replace: mamba_ssm's Mamba and the reference's CPU
    block, whichever are importable (and are not this package's class)."""
    found = []
    for modname, attr in (("mamba_ssm", "Mamba"), ("cpu_mamba", "CPUMamba")):
        mod = sys.modules.get(modname)
        if mod is None:
            try:
                mod = __import__(modname)
            except Exception:
                continue
        cls = getattr(mod, attr, None)
        if isinstance(cls, type) and cls is not CPUMamba and not issubclass(cls, CPUMamba):
            found.append(cls)
    return tuple(found)


def swap_mamba_to_b200(module: nn.Module, verbose: bool = False) -> int:
    """Replace every mamba_ssm / reference block under ``module`` by this
    package's block with the same weights (surgery.py:47-79).  Returns the
    number of blocks replaced."""
    classes = _foreign_block_classes()
    if not classes:
        return 0
    n = 0
    for name, parent in list(module.named_modules()):
        for child_name, child in list(parent.named_children()):
            if not isinstance(child, classes):
                continue
            sd = child.state_dict()
            ref = sd.get("in_proj.weight")
            block = CPUMamba(d_model=child.d_model, d_state=child.d_state, d_conv=child.d_conv,
                             expand=child.expand,
                             dt_rank=getattr(child, "dt_rank", "auto"))
            block.load_state_dict(sd, strict=True)
            if ref is not None:
                block = block.to(device=ref.device, dtype=ref.dtype)
            block.train(child.training)
            setattr(parent, child_name, block)
            n += 1
            if verbose:
                print(f"swapped {name + '.' if name else ''}{child_name}: "
                      f"{type(child).__name__} -> cpu_mamba_b200.CPUMamba")
    return n


swap_mamba_to_cpu = swap_mamba_to_b200
