"""Loader for the in-tree CUDA extension ``sigma0_b200._C``.

The extension is built in-tree (``python setup.py build_ext --inplace`` or
``__graft_entry__.build()``).  On a CUDA device the kernels are mandatory: a
missing extension raises instead of silently falling back to eager torch.

Every call through :func:`ext` is counted in kernel launches (some entry points
launch several kernels), so benchmarks can report how many of this package's
kernels ran in a timed region.
"""
from __future__ import annotations

_C = None
_COUNT = [0]
# kernels launched per call, where it is not one
_LAUNCHES = {"m3_fwd": 2, "m3_bwd": 5, "ln_bwd": 2, "rms_bwd": 2, "glu_res_bwd": 2, "attn_bwd": 2, "s5_scan_fwd": 3, "s5_scan_bwd": 3}


class _Counted:
    def __init__(self, mod):
        self._mod = mod

    def __getattr__(self, name):
        fn = getattr(self._mod, name)
        k = _LAUNCHES.get(name, 1)

        def call(*a, **kw):
            # m3_bwd skips the forward recompute (2 kernels) when given the forward's states
            _COUNT[0] += k - (2 if name == "m3_bwd" and kw.get("saved_states") is not None else 0)
            return fn(*a, **kw)
        return call


def ext():
    global _C
    if _C is None:
        try:
            from .. import _C as mod  # type: ignore
        except ImportError as e:  # pragma: no cover - only without a build
            raise RuntimeError(
                "sigma0_b200 CUDA extension is not built; run `python setup.py build_ext --inplace`") from e
        _C = _Counted(mod)
    return _C


def available() -> bool:
    try:
        ext()
        return True
    except RuntimeError:
        return False


def reset_launch_count() -> None:
    _COUNT[0] = 0


def launch_count() -> int:
    return _COUNT[0]
