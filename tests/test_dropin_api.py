"""The drop-in contract: every public hot-path function of the reference
(tests/golden/reference_api.json, read from the reference's own modules by
tests/golden/make_golden.py) exists under the same module and name here,
with the same parameters in the same order, the same kinds and the same
defaults; the only additions allowed are keyword-only parameters with
defaults (norm_weight=, x_scale=, ...).  A caller that rebinds the
reference's module names to these modules therefore calls
every function exactly as before.  CPU only."""

import importlib
import inspect
import json
import os

import pytest

from conftest import GOLDEN

with open(os.path.join(GOLDEN, "reference_api.json")) as _f:
    REFERENCE = json.load(_f)


def resolve(qualname):
    mod_name, _, rest = qualname.partition(".")
    obj = importlib.import_module(mod_name)
    for part in rest.split("."):
        obj = getattr(obj, part)
    return obj


@pytest.mark.parametrize("qualname", sorted(REFERENCE))
def test_signature_matches_reference(qualname):
    ref = REFERENCE[qualname]
    ours = list(inspect.signature(resolve(qualname)).parameters.values())
    assert len(ours) >= len(ref), f"{qualname}: fewer parameters than the reference"
    for (name, kind, default), p in zip(ref, ours):
        assert p.name == name, f"{qualname}: parameter {p.name!r} where the reference has {name!r}"
        assert p.kind.name == kind, f"{qualname}.{name}: {p.kind.name} where the reference has {kind}"
        ours_default = None if p.default is inspect.Parameter.empty else repr(p.default)
        assert ours_default == default, f"{qualname}.{name}: default {ours_default} vs the reference's {default}"
    for p in ours[len(ref):]:
        assert p.kind in (inspect.Parameter.KEYWORD_ONLY, inspect.Parameter.VAR_KEYWORD) or \
            p.default is not inspect.Parameter.empty, f"{qualname}: added parameter {p.name!r} is required"
        if p.kind is inspect.Parameter.KEYWORD_ONLY:
            assert p.default is not inspect.Parameter.empty, f"{qualname}: added {p.name!r} has no default"


def test_fixture_covers_the_hot_path():
    names = {q.split(".", 1)[1] for q in REFERENCE}
    for n in ("fused_rmsnorm_linear", "fused_rmsnorm_linear_fp8", "fused_tree_attention", "fused_paged_attention",
              "fused_multi_verify", "fused_verify", "RowParallelLinear.forward", "pack_scales"):
        assert n in names
