"""Drop-in name for users of the reference's ``foundry`` package: everything
is provided by ``foundry_b200``. The submodules ``foundry.graph``,
``foundry.allocation_region`` and ``foundry.ops`` exist as in the reference;
as there, the package attributes ``graph`` and ``allocation_region`` are the
context managers, not the modules."""

from . import allocation_region as _allocation_region_module  # noqa: F401
from . import graph as _graph_module  # noqa: F401
from . import ops  # noqa: F401
from foundry_b200 import *  # noqa: F401,F403,E402
from foundry_b200 import __all__  # noqa: F401,E402
