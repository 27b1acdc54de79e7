"""Loader for the compiled sm_100a extension (``rs_nanogpt_b200._C``).

The extension is built in-tree (``python setup.py build_ext --inplace``).
On a machine with a GPU the kernels are the only implementation of the hot
ops, so a missing extension is an error, never a silent fallback.
"""
import functools


@functools.lru_cache(maxsize=None)
def ext():
    try:
        from rs_nanogpt_b200 import _C
    except ImportError as e:
        raise RuntimeError(
            "rs_nanogpt_b200._C is not built; run `python setup.py build_ext --inplace`") from e
    return _C


def kernel_status(reset: bool = True) -> int:
    """Device error word of the kernels: 0 when every bounded wait completed."""
    return int(ext().kernel_status(reset))
