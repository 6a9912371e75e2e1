"""The reference's own LoRALinear / LoRAManager specification, run unchanged
against this package.

FitLLM pins its own-layout adapter module (fitllm/lora.py: ``LoRALinear``,
``LoRAManager``) with tests/test_lora_gradients.py: output shapes, frozen
base weights, A/B initialisation, scale = alpha / rank, injection by target
suffix, gradients only on A and B, the adapter-only state dict and its round
trip.  ``fitllm_b200.lora`` is meant as a drop-in for that module, so this
file loads that test module from a FitLLM checkout with ``fitllm.lora``
aliased to ``fitllm_b200.lora`` and runs every one of its test methods.

The checkout is found through the FITLLM_REFERENCE_DIR environment variable,
or at the read-only location the reference is mounted at in the build
container; without one the tests are skipped (they need no GPU).
"""
import importlib.util
import inspect
import os
import sys
import types

import pytest

REF_DIR = os.environ.get("FITLLM_REFERENCE_DIR", "/root/reference")
SPEC_FILE = os.path.join(REF_DIR, "tests", "test_lora_gradients.py")


def _load_spec_module():
    import fitllm_b200.lora as mine
    alias = types.ModuleType("fitllm")
    alias.__path__ = []  # a package, so "fitllm.lora" resolves
    alias.lora = mine
    saved = {k: sys.modules.get(k) for k in ("fitllm", "fitllm.lora")}
    sys.modules["fitllm"] = alias
    sys.modules["fitllm.lora"] = mine
    try:
        spec = importlib.util.spec_from_file_location("fitllm_reference_test_lora_gradients", SPEC_FILE)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
    finally:
        for k, v in saved.items():
            if v is None:
                sys.modules.pop(k, None)
            else:
                sys.modules[k] = v
    return mod


_MOD = []


def _cases():
    if not os.path.isfile(SPEC_FILE):
        return [pytest.param(None, None, marks=pytest.mark.skip(reason="no FitLLM checkout"))]
    if not _MOD:
        _MOD.append(_load_spec_module())
    mod = _MOD[0]
    cases = []
    for cname, cls in inspect.getmembers(mod, inspect.isclass):
        if not cname.startswith("Test") or cls.__module__ != mod.__name__:
            continue
        for mname, _ in inspect.getmembers(cls, inspect.isfunction):
            if mname.startswith("test_"):
                cases.append(pytest.param(cls, mname, id=f"{cname}.{mname}"))
    return cases


@pytest.mark.parametrize("cls,method", _cases())
def test_reference_lora_spec(cls, method):
    import fitllm_b200.lora as mine
    # the spec module bound LoRALinear / LoRAManager from fitllm_b200.lora
    assert _MOD[0].LoRALinear is mine.LoRALinear and _MOD[0].LoRAManager is mine.LoRAManager
    getattr(cls(), method)()


def test_reference_spec_collected_every_method():
    """All 15 test methods of the reference spec are collected (guards against
    an import shim that silently finds nothing)."""
    if not os.path.isfile(SPEC_FILE):
        pytest.skip("no FitLLM checkout")
    assert len(_cases()) == 15
