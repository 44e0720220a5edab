"""`import quail` for programs written against fsdatalab/quail: the same names, served by quail_b200."""

from quail_b200 import *  # noqa: F401,F403
from quail_b200 import __all__  # noqa: F401
