from .collator import PadSftCollator, simple_pretrain_collator
from .data_loader import DistributedDataLoader
from .data_source import PackedDataset
from .distributed_sampler import DistributedSampler
from .synthetic import SyntheticTokens
