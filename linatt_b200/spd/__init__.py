"""SPD delta-rule kernels -- drop-in for ``kata/spd`` (``kata/spd/__init__.py``).

  flash_delta        -- DeltaKATA: SPD delta rule, time-major (kata/spd/flash_delta.py)
  flash_delta_state  -- the raw-numerator delta rule, head-major (kata/spd/chunk_state_v2.py)
  spd_state_lin      -- linear (no delta) SPD numerator, head-major (kata/spd/chunk_state_lin.py)
  spd_chunk_scan     -- normalised sum-score SPD forward, head-major (kata/spd/chunk_scan.py)

As in the reference package, the function ``flash_delta`` is re-exported under the name of its
submodule.
"""

from .chunk_scan import spd_chunk_scan
from .chunk_state_lin import spd_state_lin
from .chunk_state_v2 import flash_delta_state
from .flash_delta import flash_delta

__all__ = ["flash_delta", "flash_delta_state", "spd_state_lin", "spd_chunk_scan"]
