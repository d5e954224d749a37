from .activation_ckpt import (ActivationCheckpointWrapper, apply_activation_checkpointing,
                              is_activation_checkpointed, remove_activation_checkpointing)
from .grad_accumulator import GradAccumulator
from .grad_transform import ClipGradNorm
from .lr_schedule import create_lr_schedule
from .mixed_precision_manager import MixedPrecisionManager
from .optimizer import FusedAdamW, get_param_groups
from .param_group import ParamGroup
from .train_config import TrainConfig
from .trainer import Trainer
