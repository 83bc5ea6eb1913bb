"""SPD delta-rule kernels -- drop-in for ``kata/spd`` (``kata/spd/__init__.py``).

  flash_delta  -- DeltaKATA: O(T^2) scalar-kernel delta rule (kata/spd/flash_delta.py)

As in the reference package, the function ``flash_delta`` is re-exported under the name of its
submodule.
"""

from .flash_delta import flash_delta

__all__ = ["flash_delta"]
