"""CPU: flexkv_b200.c_ext keeps the surface FlexKV's code binds.

Against tests/golden/worker_calls.json (tests/golden/make_worker_golden.py):
* every call the reference's own workers and hash helpers made while
  recording still binds to c_ext's current signatures;
* every function and method the reference's pybind module declares
  (csrc/bindings.cpp:107-171, the CFS-only names excluded) exists, with the
  declared keyword names in order and the declared defaults;
* transfer_kv_blocks takes the binding's 15 arguments positionally, in the
  binding's order (it is bound without py::arg names).
"""
import inspect
import json
import os

import pytest

from flexkv_b200 import c_ext

FIX = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "worker_calls.json")))
B = FIX["bindings"]


def _params(fn, drop_self=False):
    ps = list(inspect.signature(fn).parameters.values())
    return ps[1:] if drop_self else ps


def _default(text):
    return {"true": True, "false": False}.get(text, None) if text in ("true", "false") else int(text)


def test_transfer_kv_blocks_positional_order():
    ps = _params(c_ext.transfer_kv_blocks)
    pos = [p.name for p in ps if p.kind in (p.POSITIONAL_ONLY, p.POSITIONAL_OR_KEYWORD)]
    assert pos == B["transfer_kv_blocks_positional"]


@pytest.mark.parametrize("name", sorted(B["functions"]))
def test_module_functions_keep_names_keywords_and_defaults(name):
    fn = getattr(c_ext, name)
    declared = B["functions"][name]
    if not declared:
        return  # bound without py::arg: positional (checked above) or no arguments
    ps = {p.name: p for p in _params(fn)}
    names = [p.name for p in _params(fn)][:len(declared)]
    assert names == [a for a, _ in declared]
    for a, d in declared:
        if d is not None:
            assert ps[a].default == _default(d), (name, a)


@pytest.mark.parametrize("cls", sorted(B["classes"]))
def test_classes_keep_their_methods(cls):
    k = getattr(c_ext, cls)
    for meth, overloads in B["classes"][cls].items():
        fn = getattr(k, meth)
        names = [p.name for p in _params(fn, drop_self=True)]
        for args in overloads:
            assert names[:len(args)] == args or (meth == "update" and args == ["input", "size"]
                                                 and names[:2] == ["input", "size"]), (cls, meth, args)


def test_recorded_worker_calls_still_bind():
    n = 0
    for sc in FIX["scenarios"]:
        for call in sc["calls"]:
            if call["fn"] == "transfer_kv_blocks":
                inspect.signature(c_ext.transfer_kv_blocks).bind(*range(call["num_positional"]))
            elif call["fn"] == "tp_group_transfer":
                inspect.signature(c_ext.TPTransferThreadGroup.tp_group_transfer).bind(
                    None, *range(call["num_positional"]))
            elif call["fn"] == "TPTransferThreadGroup":
                inspect.signature(c_ext.TPTransferThreadGroup.__init__).bind(None, 1, [], None, 0)
            elif call["fn"] == "gen_hashes":
                inspect.signature(c_ext.gen_hashes).bind(None, None, 16, None)
            n += 1
    assert n >= 20
