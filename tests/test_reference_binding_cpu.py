"""The engine's binding into SoloRT's ``_GraphQwen3Runner`` (``solort_b200.reference_binding``),
checked against the reference's own class where its source tree sits next to this repository
(the reference is pure Python and imports on a CPU; elsewhere these tests skip): the mixin
overrides exactly methods the reference defines and the runner's capture helpers call, with the
same signatures, and ``install`` makes the executors construct the engine-backed runner. The
oracle's restated runner, which the GPU tests bind to, has the reference's method signatures."""

from __future__ import annotations

import inspect
import os
import sys

import pytest

from solort_b200 import reference_binding as RB

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_SRC = os.environ.get("SOLORT_REFERENCE_SRC") or os.path.join(os.path.dirname(ROOT), "reference", "src")


@pytest.fixture(scope="module")
def cge():
    if not os.path.isfile(os.path.join(REF_SRC, "solort", "model", "cuda_graph_executor.py")):
        pytest.skip("the reference source tree is not available here")
    if REF_SRC not in sys.path:
        sys.path.insert(0, REF_SRC)
    try:
        from solort.model import cuda_graph_executor
    except Exception as exc:  # pragma: no cover
        pytest.skip(f"the reference does not import here: {exc}")
    return cuda_graph_executor


def _params(fn):
    """Parameter names, kinds and defaults (annotations aside)."""
    return [(p.name, p.kind, p.default) for p in inspect.signature(fn).parameters.values()]


def _own_methods(cls):
    return {n for n, v in vars(cls).items() if inspect.isfunction(v) and not n.startswith("__")}


def test_mixin_overrides_reference_methods_with_their_signatures(cge):
    base = cge._GraphQwen3Runner
    overrides = set(RB.BOUND_METHODS)
    assert overrides <= _own_methods(RB.EngineAttention)
    for name in overrides:
        assert name in vars(base), f"{name} is not a method of _GraphQwen3Runner"
        assert _params(getattr(RB.EngineAttention, name)) == _params(getattr(base, name)), name
    # the capture helpers of the reference call exactly these methods
    src = inspect.getsource(base)
    for caller, callee in (("_capture_prefill", "_prefill_forward"), ("_capture", "_decode_forward"),
                           ("verify", "_verify_forward")):
        assert f"self.{callee}(" in inspect.getsource(getattr(base, caller)), (caller, callee)
    assert "_prefill_forward" in src
    # helper methods the mixin adds do not shadow anything of the reference
    extra = _own_methods(RB.EngineAttention) - overrides
    assert not (extra & set(dir(base))), extra & set(dir(base))
    assert _params(RB.EngineAttention.__init__) == _params(base.__init__)


def test_install_makes_the_executors_build_engine_runners(cge):
    original = cge._GraphQwen3Runner
    try:
        cls = RB.install(cge)
        assert cge._GraphQwen3Runner is cls and issubclass(cls, original)
        assert issubclass(cls, RB.EngineAttention)
        assert RB.install(cge) is cls  # idempotent
        # both executors construct the runner through the module-level name
        for ex in (cge.CudaGraphQwen3Executor, cge.SpecCudaGraphQwen3Executor):
            assert "_GraphQwen3Runner(" in inspect.getsource(ex.__init__), ex
        # the MRO puts the engine's methods first, the reference's for everything else
        for name in RB.BOUND_METHODS:
            assert getattr(cls, name) is getattr(RB.EngineAttention, name)
        for name in ("prefill", "decode", "decode_argmax", "decode_gpu", "decode_gpu_argmax",
                     "verify", "_capture", "_capture_prefill", "_replay"):
            assert getattr(cls, name) is getattr(original, name), name
    finally:
        cge._GraphQwen3Runner = original


def test_oracle_runner_has_the_reference_surface(cge):
    from oracle.runner import ReferenceQwen3Runner

    base = cge._GraphQwen3Runner
    for name in ("_cos_sin", "_rope", "_prefill_forward", "_decode_forward", "_verify_forward",
                 "prefill", "decode", "decode_argmax", "decode_gpu", "decode_gpu_argmax", "verify",
                 "_bucket_for", "_capture", "_capture_prefill"):
        want = inspect.signature(getattr(base, name))
        got = inspect.signature(getattr(ReferenceQwen3Runner, name))
        assert list(got.parameters)[:len(want.parameters)] == list(want.parameters), name
