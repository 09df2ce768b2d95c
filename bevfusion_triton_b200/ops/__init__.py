"""Operator modules with the reference's import paths (``ops.bev_pool``,
``ops.voxel``) re-rooted under this package."""
