"""ytm_b200 — a B200-native Tsetlin Machine engine with the API of
Mayur1009/YTM's `cutm` package.

    from ytm_b200.cutm import MultiClassTM, MultiOutputTM
"""
__version__ = "0.1.0"
