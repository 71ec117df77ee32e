"""Limit-order-book environments on the batched matching engine, baselines and PPO."""
from .lob_env import (BaseLOBEnv, MarketMakingEnv, ExecutionEnv, MultiAgentEnv, EnvWindow, windows_from_days,
                      features)

__all__ = ["BaseLOBEnv", "MarketMakingEnv", "ExecutionEnv", "MultiAgentEnv", "EnvWindow", "windows_from_days",
           "features"]
