"""The drop-in binding (maskahead_b200.dropin) against the reference package itself.

Every operator the shim rebinds keeps the reference's signature (each call shape the
reference accepts, ours accepts), install() reaches every call site -- the module that
defines each name and the modules that imported it by name (runtime/session.py:14-21,
kernels/__init__.py:1-7) -- and uninstall() puts the reference's objects back. Skipped
when the reference package is not importable (tests/reference_pkg.py).
"""

from __future__ import annotations

import importlib
import sys

import pytest

from reference_pkg import reference_package

REF = reference_package()
pytestmark = pytest.mark.skipif(REF is None, reason="reference package not installed (baseline/_ref)")


def _pairs():
    from maskahead_b200.dropin import BINDINGS

    for ref_mod, name, our_mod, our_name, _scope in BINDINGS:
        yield (f"{ref_mod}.{name}", getattr(importlib.import_module(f"maskahead.{ref_mod}"), name),
               getattr(importlib.import_module(our_mod), our_name))


def test_every_binding_accepts_the_reference_calls():
    from maskahead_b200.dropin import signature_gaps

    gaps = {label: g for label, ref, ours in _pairs() if (g := signature_gaps(ref, ours))}
    assert not gaps, gaps


def test_prefix_and_selector_result_carry_the_reference_fields():
    from maskahead.kernels import ops as rops
    from maskahead.kernels import splitk as rsplitk

    from maskahead_b200.kernels import SelectorResult
    from maskahead_b200.layouts import Prefix

    assert set(rsplitk.Prefix.__slots__) <= set(Prefix.__slots__)
    assert isinstance(Prefix.n, property)
    ref_fields = set(rops.SelectorResult.__dataclass_fields__)
    assert ref_fields <= set(SelectorResult.__dataclass_fields__)


def test_install_rebinds_every_call_site_and_uninstall_restores():
    from maskahead_b200 import dropin

    originals = {label: ref for label, ref, _ in _pairs()}
    session = sys.modules["maskahead.runtime.session"]
    kernels = sys.modules["maskahead.kernels"]
    inst = dropin.install()
    try:
        for label, _ref, ours in _pairs():
            mod, name = label.rsplit(".", 1)
            assert getattr(sys.modules[f"maskahead.{mod}"], name) is ours, label
        from maskahead_b200.kernels import ops as bops
        from maskahead_b200.kernels import splitk as bsplitk

        # names the session bound at import, and the kernels package's re-exports
        for name in ("selector_topk", "gather_packed_kv", "dense_packed_attention"):
            assert getattr(session, name) is getattr(bops, name)
            assert getattr(kernels, name) is getattr(bops, name)
        assert session.sdpa_compact is bops.sdpa_compact
        assert sys.modules["maskahead.reference"].sdpa_compact is originals["runtime.session.sdpa_compact"]
        # the fast path imports splitk names inside its methods: they resolve to ours
        from maskahead.kernels.splitk import Prefix, prefix_scores, splitk_attention

        assert (Prefix, prefix_scores, splitk_attention) == (bsplitk.Prefix, bsplitk.prefix_scores,
                                                             bsplitk.splitk_attention)
        with pytest.raises(RuntimeError):
            dropin.install()
    finally:
        inst.uninstall()
    for label, ref, _ in _pairs():
        assert ref is originals[label], label
    assert session.selector_topk is originals["kernels.ops.selector_topk"]
    assert kernels.gather_packed_kv is originals["kernels.ops.gather_packed_kv"]
    dropin.install().uninstall()          # installable again after uninstall
