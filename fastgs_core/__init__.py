"""Import-compatible alias of the reference package name.

Training scripts written against the reference do ``import fastgs_core`` or
``from fastgs_core import _fastgs_core``; both resolve to fastgs_core_b200.
"""
from fastgs_core_b200 import *  # noqa: F401,F403
from fastgs_core_b200 import api as _fastgs_core  # noqa: F401
