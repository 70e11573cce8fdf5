"""Loader for the sm_100a extension ``nexttransformer_b200._C``.

CUDA tensors always go through these kernels.  If the library is missing on a machine with a
GPU, every op raises instead of silently running a slower PyTorch path; CPU tensors use the
plain-PyTorch restatement of each op (the oracle the kernels are tested against).
"""
import importlib

_lib = None
_err = None


def ext():
    """Return the compiled extension module or raise with build instructions."""
    global _lib, _err
    if _lib is None and _err is None:
        try:
            _lib = importlib.import_module("nexttransformer_b200._C")
        except ImportError as e:  # pragma: no cover - depends on the build
            _err = e
    if _lib is None:
        raise RuntimeError("nexttransformer_b200._C is not built; run `python -m nexttransformer_b200.build` "
                           f"({_err})")
    return _lib


def available():
    try:
        ext()
        return True
    except RuntimeError:
        return False


def check_errors():
    """Raise if a bounded device-side wait in a kernel gave up (see csrc/common.cuh)."""
    g, gw, a, aw, d, dw, sp, sw = ext().read_errors()
    if g or a or d or sp:
        raise RuntimeError(f"device pipeline wait expired: gemm code {g} at {gw:#x}, attention code {a} at {aw:#x}, "
                           f"delta scan code {d} at {dw:#x}, sparse attention code {sp} at {sw:#x}")
