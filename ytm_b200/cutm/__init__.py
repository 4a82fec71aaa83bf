"""Drop-in for the reference's `cutm` package (src/cutm/__init__.py:1-2)."""
from .base import BaseTM as BaseTM
from .multiclass import MultiClassTM as MultiClassTM
from .multioutput import MultiOutputTM as MultiOutputTM
