"""Book-state world model (frames on a wall clock, chart representation, DiT, flow matching)."""
from .model import (BookDiT, decode_chart, encode_chart, flow_matching_loss, resample_frames, reward_weighted_loss,
                    sample, smoothness_reward, spread_reward)

__all__ = ["BookDiT", "decode_chart", "encode_chart", "flow_matching_loss", "resample_frames",
           "reward_weighted_loss", "sample", "smoothness_reward", "spread_reward"]
