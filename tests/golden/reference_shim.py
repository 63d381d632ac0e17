"""Import shim that lets the SpecFit reference be imported in a container
without its two absent third-party packages.

Used by ``make_golden.py`` (fixture generation) and by the CPU test that
constructs the reference speculator around this package's model
(``tests/test_attention_install.py``), both run where the reference source
tree is present.  Nothing on the product path imports it.

* ``speculators`` 0.5.0 (pinned by the reference's requirements-test.txt:8)
  supplies the EAGLE-3 drafter; the reference imports it in
  ``src/specfit/runtime/eagle3_chain.py:11`` and ``eagle3_attention.py:5-11``.
  Only names are needed here, never behaviour.
* ``accelerate`` 1.14.0 (requirements-test.txt:7) is imported by
  ``src/specfit/runtime/qwen3_offloaded_model.py:15-16``.  It must be
  injected *after* ``transformers`` has been imported, otherwise
  transformers' own version probe of accelerate fails.
"""
from __future__ import annotations

import contextlib
import sys
import types


def _module(name: str, **attrs) -> types.ModuleType:
    module = types.ModuleType(name)
    for key, value in attrs.items():
        setattr(module, key, value)
    sys.modules.setdefault(name, module)
    return sys.modules[name]


class _Registry(dict):
    def register(self, key, value):
        self[key] = value


def _unavailable(*_args, **_kwargs):
    raise NotImplementedError("speculators is not installed; import-only shim")


class _Eagle3DraftModel:  # import-only placeholder
    pass


def install(reference_src: str) -> None:
    """Make ``import specfit`` work from ``reference_src`` (its ``src`` dir)."""
    import transformers  # noqa: F401  (real import before the accelerate shim)
    from transformers import Qwen3MoeConfig, Qwen3MoeForCausalLM  # noqa: F401

    _module("speculators")
    _module("speculators.models")
    _module(
        "speculators.models.attention",
        ALL_ATTENTION_FUNCTIONS=_Registry(),
        flex_attention_forward=_unavailable,
    )
    _module("speculators.models.eagle3", Eagle3DraftModel=_Eagle3DraftModel)
    _module("speculators.models.eagle3.core", extend_mask_for_draft_tokens=_unavailable)
    _module(
        "speculators.models.eagle3.attention",
        extend_mask_for_draft_tokens=_unavailable,
    )
    sys.modules["speculators.models.eagle3"].core = sys.modules["speculators.models.eagle3.core"]
    sys.modules["speculators.models.eagle3"].attention = sys.modules[
        "speculators.models.eagle3.attention"
    ]

    @contextlib.contextmanager
    def init_empty_weights(include_buffers: bool = False):
        import torch

        with torch.device("meta"):
            yield

    def set_module_tensor_to_device(module, name, device, value=None, dtype=None, clear_cache=False):
        import torch

        *path, leaf = name.split(".")
        owner = module
        for part in path:
            owner = getattr(owner, part)
        old = getattr(owner, leaf)
        tensor = value.to(device=device, dtype=dtype or value.dtype)
        if isinstance(old, torch.nn.Parameter):
            tensor = torch.nn.Parameter(tensor, requires_grad=False)
        setattr(owner, leaf, tensor)

    utils = _module("accelerate.utils", set_module_tensor_to_device=set_module_tensor_to_device)
    _module("accelerate", __version__="1.14.0", init_empty_weights=init_empty_weights, utils=utils)
    if reference_src not in sys.path:
        sys.path.insert(0, reference_src)
