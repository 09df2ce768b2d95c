from .bev_pool import bev_pool, bev_pool_depth_context, bev_pool_plan, bev_pool_planned

__all__ = ['bev_pool', 'bev_pool_depth_context', 'bev_pool_plan', 'bev_pool_planned']
