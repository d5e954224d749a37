"""Materialise a meta-device model into packed per-unit parameter storage.

Every unit (by default each LlamaDecoderLayer, and one unit for everything else) receives
one contiguous bf16 allocation and its parameters become views into it, in registration
order.  This keeps q|k|v and gate|up consecutive, so the fused GEMMs use them as one operand
without copies, and lets optimizer / sharding code treat a unit as a single flat buffer.

Random initialisation mirrors the reference CLI (femtotron/scripts/train.py:213-219): every
parameter, in ``model.parameters()`` order, is drawn from N(0, init_std) in fp32 on the
target device and then cast to the compute dtype, so a given seed gives the same weights as
the reference path.
"""
from __future__ import annotations

from typing import Callable

import torch
from torch import nn

from .layers import LlamaDecoderLayer


def default_unit_policy(m: nn.Module) -> bool:
    return isinstance(m, LlamaDecoderLayer)


def _owner_map(model: nn.Module):
    owners = {}
    for mname, mod in model.named_modules():
        for pname, p in mod.named_parameters(recurse=False):
            owners.setdefault(id(p), []).append((mod, pname))
    return owners


def materialize_model(model: nn.Module, device, dtype=torch.bfloat16, init_std: float | None = 0.02,
                      unit_policy: Callable[[nn.Module], bool] = default_unit_policy,
                      init_fn: Callable[[str, torch.Tensor], None] | None = None) -> nn.Module:
    device = torch.device(device)
    owners = _owner_map(model)
    units = [m for m in model.modules() if unit_policy(m)]
    seen: set[int] = set()
    groups: list[list[nn.Parameter]] = []
    for u in units:
        ps = []
        for p in u.parameters():
            if id(p) not in seen:
                seen.add(id(p))
                ps.append(p)
        if ps:
            groups.append(ps)
    rest = []
    for p in model.parameters():
        if id(p) not in seen:
            seen.add(id(p))
            rest.append(p)
    for p in rest:
        groups.append([p])

    new_of: dict[int, nn.Parameter] = {}
    for ps in groups:
        total = sum(p.numel() for p in ps)
        flat = torch.empty(total, dtype=dtype, device=device)
        off = 0
        for p in ps:
            view = flat[off:off + p.numel()].view(p.shape)
            off += p.numel()
            newp = nn.Parameter(view, requires_grad=p.requires_grad)
            new_of[id(p)] = newp
            for mod, pname in owners[id(p)]:
                mod._parameters[pname] = newp
    # non-parameter buffers (none are persistent in the LLaMA model) follow the device
    for mod in model.modules():
        for bname, b in list(mod._buffers.items()):
            if b is not None and b.device.type == "meta":
                mod._buffers[bname] = torch.zeros(b.shape, dtype=b.dtype, device=device)
    # initialisation, in model.parameters() order (tied weights once)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if init_fn is not None:
                init_fn(name, p)
            elif init_std is not None:
                tmp = torch.empty(p.shape, dtype=torch.float32, device=device)
                tmp.normal_(mean=0.0, std=init_std)
                p.copy_(tmp)
    return model
