"""Launch handles that keep the reference's ``kernel[grid](...)`` call form.

The reference exports its ``@triton.jit`` kernels and its tests launch them as
``kernel[(N_rows,)](tensor args..., name=value..., BLOCK_V=..., num_warps=...)``
(``solution/test_kernels.py:125-138``). A :class:`LaunchShim` accepts the same
positional/keyword arguments, maps them to one C-ABI call and ignores the
Triton-only tuning keywords (block sizes, ``num_warps``, ``num_stages``); the
grid is chosen by the CUDA side.
"""

from __future__ import annotations


class LaunchShim:
    def __init__(self, name, params, launch):
        self.__name__ = name
        self._params = list(params)
        self._launch = launch

    def __getitem__(self, grid):
        def run(*args, **kwargs):
            if len(args) > len(self._params):
                raise TypeError(f"{self.__name__}: too many positional arguments")
            bound = dict(zip(self._params, args))
            for k, v in kwargs.items():
                if k in bound:
                    raise TypeError(f"{self.__name__}: argument {k!r} given twice")
                bound[k] = v
            missing = [p for p in self._params if p not in bound]
            if missing:
                raise TypeError(f"{self.__name__}: missing arguments {missing}")
            return self._launch(**bound)

        return run

    def __repr__(self):
        return f"<sm_100a kernel {self.__name__}>"
