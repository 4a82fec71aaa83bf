"""Drop-in for the reference's CPU Tsetlin Machine package `pytm`
(src/pytm/base.py), running on the B200 engine:

    from ytm_b200.pytm.base import BaseTM
"""
from .base import BaseTM as BaseTM
