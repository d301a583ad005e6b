"""Memory substrate and bundle grouping for verification."""

from .bundle_scheduler import BundleScheduler, TreeDescriptorBuilder

__all__ = ["BundleScheduler", "TreeDescriptorBuilder"]
