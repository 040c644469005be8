"""Import path kept from the reference (``minisgl.distributed``); the code lives in
``minisgl.parallel``."""

from minisgl.parallel import *  # noqa: F401,F403
from minisgl.parallel import __all__  # noqa: F401
