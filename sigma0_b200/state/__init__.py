"""Book-state world model: wall-clock frames, chart coordinates, DiT velocity models,
rectified flow, rewards and post-training (the reference's ``src/state`` package)."""
from .dit import FrameDiT, FrameDiTConfig, bind_condition, bind_unconditional
from .flow import (RectifiedFlow, SdeStepRecord, eps_from_v, fm_loss, interpolate, make_repaint_pin,
                   score_from_v, velocity_target, x0_from_v)
from .frames import DEFAULT_INTERVAL_NS, FrameSeries, absolute_time_ns, resample_events, resample_frames, \
    resample_wide_book
from .model import BookDiT, bind_bookdit, flow_matching_loss, sample
from .posttraining import (AWMTrainer, DMDRTrainer, DMDTrainer, FlowGRPOTrainer, RAMTrainer, ReFLTrainer,
                           group_advantage)
from .representation import ChartNormalizer, chart_channels, decode_frames, decode_frames_torch, encode_frames
from .rewards import (BookValidityReward, CompositeReward, ReturnSanityReward, SpreadBandReward,
                      default_rule_reward, smoothness_reward, spread_reward)
from .train import (EncodedDay, FrameWindowDataset, encode_series, fit_normalizer, load_checkpoint,
                    pretrain_step, sample_context_masks, save_checkpoint)
