"""SPD delta-rule kernels -- drop-in for ``kata/spd`` (``kata/spd/__init__.py``).

  flash_delta        -- DeltaKATA: SPD delta rule, time-major (kata/spd/flash_delta.py)
  flash_delta_state  -- the raw-numerator delta rule, head-major (kata/spd/chunk_state_v2.py)

As in the reference package, the function ``flash_delta`` is re-exported under the name of its
submodule.
"""

from .chunk_state_v2 import flash_delta_state
from .flash_delta import flash_delta

__all__ = ["flash_delta", "flash_delta_state"]
