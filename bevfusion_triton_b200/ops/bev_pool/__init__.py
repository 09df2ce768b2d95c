from .bev_pool import (bev_grid, bev_pool, bev_pool_depth_context, bev_pool_geometry_plan, bev_pool_plan,
                       bev_pool_planned, check_plan, plan_matches)

__all__ = ['bev_grid', 'bev_pool', 'bev_pool_depth_context', 'bev_pool_geometry_plan', 'bev_pool_plan',
           'bev_pool_planned', 'check_plan', 'plan_matches']
