"""Drop-in name for users of the reference's ``foundry`` package: everything
is provided by ``foundry_b200``."""
from foundry_b200 import *  # noqa: F401,F403
from foundry_b200 import __all__  # noqa: F401
