from .action import (Backward, Forward, PPAction, RecvBackward, RecvForward, SendBackward,
                     SendBackwardRecvForward, SendForward, SendForwardRecvBackward)
from .comm_ops import PipelineComm
from .microbatch import split_microbatches
from .partition import partition_layers
from .pipeline_config import PipelineConfig
from .runner import PipelineRunner
from .schedule import gpipe_schedule, one_f_one_b_schedule
from .stage import PipelineStage
