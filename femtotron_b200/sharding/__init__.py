from .cluster_sharding_spec import ClusterShardingSpec, compute_cluster_layout
from .factory import create_sharding_strategy
from .no_shard import NoShardStrategy
from .param_group_cluster import ParamGroupCluster
from .sharding_spec import ShardingSpec
from .wrap_policy import llama_wrap_policy, make_class_wrap_policy
from .zero1 import ZeRO1Strategy
from .zero2 import ZeRO2Strategy
from .zero3 import ZeRO3Strategy
from .zero_config import ZeROConfig
