"""Binding the sm_100a operators into the reference package at run time.

``install()`` is the shim a maintainer of the reference adds (behind a switch, e.g. in
src/maskahead/kernels/__init__.py): it rebinds the reference's operator names to this
package's implementations -- in the module that defines each one and in every module of
the package that imported it by name (runtime/session.py:14-21 binds the ops names when
it is imported; kernels/__init__.py:1-7 re-exports them; the fast path imports the
splitk names inside its methods, runtime/session.py:1363, 1381, 1396, 1406). The
reference's own call sites then run the sm_100a kernels with their arguments unchanged:
step 0 of a block, the dense layers, the probes and the sub-steps of its fast path
(runtime/session.py:1286-1459, 2254-2418) and the cache's quantizers (cache.py:482-540).

    reference name                        defined at                  rebound in
    kernels.ops.selector_topk             kernels/ops.py:790-832      the package
    kernels.ops.gather_packed_kv          kernels/ops.py:835-855      the package
    kernels.ops.dense_packed_attention    kernels/ops.py:766-787      the package
    kernels.ops.quantize_key_groups_into  kernels/ops.py:665-712      the package
    kernels.ops.quantize_values_into      kernels/ops.py:715-763      the package
    kernels.splitk.splitk_attention       kernels/splitk.py:493-579   the package
    kernels.splitk.prefix_scores          kernels/splitk.py:582-614   the package
    kernels.splitk.dequantize_prefix      kernels/splitk.py:465-480   the package
    kernels.splitk.Prefix                 kernels/splitk.py:408-462   the package
    runtime.session.sdpa_compact          reference.py:403-426        runtime/session.py only
    runtime.session.value_score           runtime/session.py:27-40    runtime/session.py only

sdpa_compact is rebound in the session alone (the model adapters keep torch's attention
for their own tensors). value_score computes its centre in fp32 where the reference's
computes it in the values' dtype (bf16), the centre its fast path's prefix_scores uses.

The operators have no CPU path: after install() the package's CPU sessions cannot run
their slow path (the operators raise KernelUnavailableError on host tensors); uninstall()
puts the reference's objects back.
"""

from __future__ import annotations

import importlib
import inspect
import sys
from dataclasses import dataclass, field

__all__ = ["BINDINGS", "Installation", "install", "signature_gaps"]

# (reference module, name, our module, our name, scope): scope "package" rebinds every
# module of the package that holds the reference's object; "module" only the first.
BINDINGS = (
    ("kernels.ops", "selector_topk", "maskahead_b200.kernels.ops", "selector_topk", "package"),
    ("kernels.ops", "gather_packed_kv", "maskahead_b200.kernels.ops", "gather_packed_kv", "package"),
    ("kernels.ops", "dense_packed_attention", "maskahead_b200.kernels.ops", "dense_packed_attention", "package"),
    ("kernels.ops", "quantize_key_groups_into", "maskahead_b200.kernels.ops", "quantize_key_groups_into",
     "package"),
    ("kernels.ops", "quantize_values_into", "maskahead_b200.kernels.ops", "quantize_values_into", "package"),
    ("kernels.splitk", "splitk_attention", "maskahead_b200.kernels.splitk", "splitk_attention", "package"),
    ("kernels.splitk", "prefix_scores", "maskahead_b200.kernels.splitk", "prefix_scores", "package"),
    ("kernels.splitk", "dequantize_prefix", "maskahead_b200.kernels.splitk", "dequantize_prefix", "package"),
    ("kernels.splitk", "Prefix", "maskahead_b200.layouts", "Prefix", "package"),
    ("runtime.session", "sdpa_compact", "maskahead_b200.kernels.ops", "sdpa_compact", "module"),
    ("runtime.session", "value_score", "maskahead_b200.hotpath", "value_score", "module"),
)

_INSTALLED: dict[str, "Installation"] = {}


@dataclass
class Installation:
    """What install() rebound: (module, name, the reference's object) per rebinding."""

    package: str
    rebound: list = field(default_factory=list)

    def uninstall(self) -> None:
        for mod, name, original in reversed(self.rebound):
            setattr(mod, name, original)
        self.rebound.clear()
        _INSTALLED.pop(self.package, None)


def install(package: str = "maskahead") -> Installation:
    """Rebind the reference package's operators (BINDINGS) to the sm_100a ones.

    Loads the kernel library first, so a missing build fails here rather than inside a
    generation (a missing CUDA device fails at the first operator call). Installing twice
    into one package raises."""
    from ._lib import load_library

    if package in _INSTALLED:
        raise RuntimeError(f"maskahead_b200 is already installed into {package!r}")
    load_library()
    inst = Installation(package)
    try:
        for ref_mod, name, our_mod, our_name, scope in BINDINGS:
            home = importlib.import_module(f"{package}.{ref_mod}")
            original = getattr(home, name)
            ours = getattr(importlib.import_module(our_mod), our_name)
            if scope == "module":
                mods = [home]
            else:
                mods = [m for key, m in list(sys.modules.items())
                        if m is not None and (key == package or key.startswith(package + "."))]
            for mod in mods:
                if mod.__dict__.get(name) is original:
                    inst.rebound.append((mod, name, original))
                    setattr(mod, name, ours)
    except Exception:
        inst.uninstall()
        raise
    _INSTALLED[package] = inst
    return inst


def _call_forms(sig: inspect.Signature):
    """The call shapes a signature accepts: everything positional that can be, every
    name that can be, and the required parameters alone."""
    P = inspect.Parameter
    params = [p for p in sig.parameters.values() if p.kind not in (P.VAR_POSITIONAL, P.VAR_KEYWORD)]
    kw_only = {p.name: None for p in params if p.kind == P.KEYWORD_ONLY}
    pos = [p.name for p in params if p.kind in (P.POSITIONAL_ONLY, P.POSITIONAL_OR_KEYWORD)]
    pos_only = [p.name for p in params if p.kind == P.POSITIONAL_ONLY]
    named = {p.name: None for p in params if p.kind in (P.POSITIONAL_OR_KEYWORD, P.KEYWORD_ONLY)}
    req_pos = [p.name for p in params if p.default is P.empty and p.kind in (P.POSITIONAL_ONLY,
                                                                             P.POSITIONAL_OR_KEYWORD)]
    req_kw = {p.name: None for p in params if p.default is P.empty and p.kind == P.KEYWORD_ONLY}
    return (("positional", pos, kw_only), ("by name", pos_only, named), ("required only", req_pos, req_kw))


def signature_gaps(reference, ours) -> list[str]:
    """Calls the reference's callable accepts that ours rejects (empty: a drop-in).

    For a class, its constructor and its public classmethods are compared."""
    if inspect.isclass(reference):
        gaps = [f"__init__: {g}" for g in signature_gaps(reference.__init__, ours.__init__)]
        for attr, obj in vars(reference).items():
            if isinstance(obj, classmethod) and not attr.startswith("_"):
                if not hasattr(ours, attr):
                    gaps.append(f"{attr}: missing")
                    continue
                gaps += [f"{attr}: {g}" for g in signature_gaps(getattr(reference, attr), getattr(ours, attr))]
        return gaps
    want, have = inspect.signature(reference), inspect.signature(ours)
    gaps = []
    for what, args, kwargs in _call_forms(want):
        try:
            have.bind(*args, **kwargs)
        except TypeError as e:
            gaps.append(f"{what} call {args} {sorted(kwargs)}: {e}")
    return gaps
