"""Closed-loop market-making simulation against replayed or generated order flow."""
from .mm_sim import Episode, EpisodeResult, build_episodes, run_episodes, autopsy

__all__ = ["Episode", "EpisodeResult", "build_episodes", "run_episodes", "autopsy"]
