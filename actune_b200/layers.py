"""Install a calibrated resident bank into an existing PyTorch backbone.

Drop-in for the reference's actune/layers.py:9-91: ``tensor_storage_bytes``,
``ResidentLinear``, ``BankRuntime`` and ``install_bank(model, bank, clips, *,
channel_scales=None, tune=False)`` with the same validation order and
ValueError messages.  The backend buffers keep the reference's names, shapes
and dtypes, so a bank's ``version_bytes`` (calibrated against the reference)
match these backends byte for byte.
"""
from __future__ import annotations

from types import MethodType

import torch

from .kernels.grouped import GroupedPaddedLinear


def tensor_storage_bytes(module):
    """Bytes of distinct storages behind the module's parameters and buffers."""
    seen, total = set(), 0
    for tensor in list(module.parameters()) + list(module.buffers()):
        storage = tensor.untyped_storage()
        key = (tensor.device, storage.data_ptr())
        if key not in seen:
            seen.add(key)
            total += storage.nbytes()
    return total


class ResidentLinear(GroupedPaddedLinear):
    """A GroupedPaddedLinear with an optional per-input-channel runtime scale.

    With ``input_scale`` the weight is multiplied by the scale before
    quantization and every input is divided by it (reference layers.py:20-43)."""

    def __init__(self, linear, assignments, clips, input_scale=None):
        if input_scale is not None:
            scale = torch.as_tensor(input_scale, device=linear.weight.device, dtype=linear.weight.dtype)
            if scale.shape != (linear.in_features,) or not torch.isfinite(scale).all() or not (scale > 0).all():
                raise ValueError("Invalid calibrated channel scale")
            scaled = torch.nn.Linear(linear.in_features, linear.out_features, bias=linear.bias is not None,
                                     device=linear.weight.device, dtype=linear.weight.dtype)
            with torch.no_grad():
                scaled.weight.copy_(linear.weight * scale[None, :])
                if linear.bias is not None:
                    scaled.bias.copy_(linear.bias)
            linear = scaled
        else:
            scale = None
        super().__init__(linear, assignments, "q11", clips)
        self.register_buffer("input_scale", scale)

    def forward(self, value):
        if self.input_scale is not None:
            value = value / self.input_scale
        return super().forward(value)


class BankRuntime:
    def __init__(self, bank, modules):
        self.bank, self.modules = bank, modules

    def before(self):
        for module in self.modules.values():
            module.calls = module.input_elements = 0

    def audit(self, configuration):
        counts = {name: module.input_elements for name, module in self.modules.items()}
        return self.bank.check_request(configuration, counts)

    def decode_weights(self):
        """Keep int8 weight codes beside every packed sub-byte version, used by calls
        of more than 32 token rows (bit-identical outputs, faster tile GEMM); returns
        the device bytes added.  The bank's storage accounting covers the packed
        versions only."""
        from .kernels.grouped import decode_weights
        return sum(decode_weights(module) for module in self.modules.values())


def install_bank(model, bank, clips, *, channel_scales=None, tune=False):
    """Replace every bank target of ``model`` with a ResidentLinear (all nine W/A pairs).

    Checks, before touching the model: bank validity, that each target is an
    nn.Linear of the calibrated shape, that each built backend's storage equals
    the bank's ``version_bytes``, and the total storage budget.  ``tune=True``
    lets each backend pick its fastest bit-identical tile variant on first use."""
    bank.validate()
    scales = {} if channel_scales is None else channel_scales
    originals = {name: model.get_submodule(name) for name in bank.shapes}
    for name, module in originals.items():
        if not isinstance(module, torch.nn.Linear) or [module.out_features, module.in_features] != list(bank.shapes[name]):
            raise ValueError(f"Target does not match the calibrated matrix: {name}")
    replacements = {}
    for name, linear in originals.items():
        assignments = {q: c[name] for q, c in bank.configurations.items()}
        replacement = ResidentLinear(linear, assignments, clips[name], scales.get(name))
        for mode, backend in replacement.backends.items():
            if tensor_storage_bytes(backend) != bank.version_bytes[name][mode]:
                raise ValueError(f"Loaded backend storage differs from calibration: {name}/{mode}")
            if tune:
                from .kernels.tuning import grouped_forward
                backend._untuned_forward = backend.forward
                backend.forward = MethodType(grouped_forward, backend)
        replacements[name] = replacement
    if sum(tensor_storage_bytes(m) for m in replacements.values()) > bank.storage_limit:
        raise ValueError("Loaded bank, including channel scales, exceeds storage budget")
    for name, module in replacements.items():
        parent, _, child = name.rpartition(".")
        setattr(model.get_submodule(parent), child, module)
    return BankRuntime(bank, replacements)


def expected_version_bytes(out_features, in_features, w, a, bias_dtype=None):
    """Storage bytes of one GroupedLinear backend: packed weight + f32 row scales (+ bias),
    with K padded to a multiple of 128 as GroupedPaddedLinear does."""
    k = (in_features + 127) // 128 * 128
    size = out_features * k * w // 8 + 4 * out_features
    if bias_dtype is not None:
        size += out_features * (4 if a == 4 else torch.empty(0, dtype=bias_dtype).element_size())
    return size
