"""Loader for the compiled sm_100a extension (``rs_nanogpt_b200._C``).

The extension is built in-tree (``python setup.py build_ext --inplace``).
On a machine with a GPU the kernels are the only implementation of the hot
ops, so a missing extension is an error, never a silent fallback.

Every call into the extension goes through a counting proxy, so callers such
as ``bench.py`` can report how many of this package's kernels were launched
(``launch_count``).
"""
import functools

# Kernels launched per extension call (1 unless listed; a callable gets the
# call's arguments).
_LAUNCHES = {"flash_bwd": 3, "flash_bwd_tc": lambda *a, **k: 2 if (a[-1] is True or k.get("prepared")) else 3,
             "flash_bwd_prep": 1, "kernel_status": 0, "flash_fwd_tc_supported": 0,
             "flash_bwd_tc_supported": 0, "flash_bwd_trace": 0, "gemm_trace": 0, "set_pdl": 0,
             "decode_attention": lambda qkv, kc, vc, pos, out, po, pm, chunk: 1 + int(kc.shape[2] > chunk)}
_count = [0]


class _Counted:
    def __init__(self, mod):
        self._mod = mod

    def __getattr__(self, name):
        fn = getattr(self._mod, name)
        n = _LAUNCHES.get(name, 1)

        def call(*args, **kwargs):
            _count[0] += n(*args, **kwargs) if callable(n) else n
            return fn(*args, **kwargs)

        return call


@functools.lru_cache(maxsize=None)
def ext():
    try:
        from rs_nanogpt_b200 import _C
    except ImportError as e:
        raise RuntimeError(
            "rs_nanogpt_b200._C is not built; run `python setup.py build_ext --inplace`") from e
    return _Counted(_C)


def launch_count() -> int:
    return _count[0]


def kernel_status(reset: bool = True) -> int:
    """Device error word of the kernels: 0 when every bounded wait completed."""
    return int(ext().kernel_status(reset))
