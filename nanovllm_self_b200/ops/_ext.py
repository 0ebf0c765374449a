"""Loader of the in-tree CUDA extension ``nanovllm_self_b200._C`` (sm_100a kernels).

There is deliberately no fallback: on a GPU, a missing or stale extension is an error
that names the build command.
"""
from __future__ import annotations

_C = None


def load():
    global _C
    if _C is None:
        try:
            from .. import _C as ext  # type: ignore[attr-defined]
        except ImportError as e:  # pragma: no cover - depends on the build
            raise RuntimeError(
                "nanovllm_self_b200._C (the sm_100a kernels) is not built: run "
                "`python setup.py build_ext --inplace` in the repository root") from e
        _C = ext
    return _C


def available() -> bool:
    try:
        load()
        return True
    except RuntimeError:
        return False
