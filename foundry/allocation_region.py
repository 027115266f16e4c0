"""``foundry.allocation_region``: the region helpers of the reference's
python/foundry/allocation_region.py, provided by foundry_b200."""

from foundry_b200.allocation_region import (  # noqa: F401
    allocation_region,
    free_preallocated_region,
    get_current_alloc_offset,
    parse_size,
    preallocate_region,
    release_allocation_region,
    resume_allocation_region,
    set_allocation_region,
    set_current_alloc_offset,
    stop_allocation_region,
)

__all__ = ["allocation_region", "free_preallocated_region", "get_current_alloc_offset", "parse_size",
           "preallocate_region", "release_allocation_region", "resume_allocation_region", "set_allocation_region",
           "set_current_alloc_offset", "stop_allocation_region"]
