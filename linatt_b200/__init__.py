"""linatt_b200 -- B200-native (sm_100a) KATA-SPD attention hot path of ayghri/linatt.

Drop-in modules mirroring the reference's operator API:
  linatt_b200.parallel_kata_attn   <-> kata/parallel_kata_attn.py
All compute runs in ``libkata_b200.so`` (C ABI: include/kata_b200.h); build it with
``python -m linatt_b200.build``.
"""

from ._lib import check_device_status  # noqa: F401

__all__ = ["check_device_status"]
