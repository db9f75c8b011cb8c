"""The 14 wide primitives (same names and import paths as the reference,
wide_compiler/core/primitives/__init__.py:26-107). Every forward runs on the
libwidek sm_100a kernels."""
from .wide_linear import WideLinear, LinearStrategy, select_linear_strategy, LINEAR_THRESHOLDS
from .wide_conv1d import WideConv1d, Conv1dStrategy
from .wide_conv2d import WideConv2d, ConvStrategy, select_strategy, STRATEGY_THRESHOLDS
from .wide_conv3d import WideConv3d, Conv3dStrategy
from .wide_batchnorm_1d import WideBatchNorm1d
from .wide_batchnorm_2d import WideBatchNorm2d
from .wide_layernorm import WideLayerNorm
from .wide_groupnorm import WideGroupNorm, GroupNormStrategy
from .wide_instancenorm import WideInstanceNorm1d, WideInstanceNorm2d, InstanceNormStrategy
from .wide_embedding import WideEmbedding, EmbeddingStrategy
from .wide_attention import WideAttention, AttentionStrategy
from .wide_gru import WideGRU, GRUStrategy
from .wide_lstm import WideLSTM, LSTMStrategy

# torch.nn type name -> Wide class (the registry and the tracer both use it).
BUILTIN_PRIMITIVES = {
    'Linear': WideLinear,
    'Conv1d': WideConv1d,
    'Conv2d': WideConv2d,
    'Conv3d': WideConv3d,
    'BatchNorm1d': WideBatchNorm1d,
    'BatchNorm2d': WideBatchNorm2d,
    'LayerNorm': WideLayerNorm,
    'GroupNorm': WideGroupNorm,
    'InstanceNorm1d': WideInstanceNorm1d,
    'InstanceNorm2d': WideInstanceNorm2d,
    'Embedding': WideEmbedding,
    'MultiheadAttention': WideAttention,
    'GRU': WideGRU,
    'LSTM': WideLSTM,
}

__all__ = [
    'WideLinear', 'LinearStrategy', 'select_linear_strategy', 'LINEAR_THRESHOLDS',
    'WideConv1d', 'Conv1dStrategy',
    'WideConv2d', 'ConvStrategy', 'select_strategy', 'STRATEGY_THRESHOLDS',
    'WideConv3d', 'Conv3dStrategy',
    'WideBatchNorm1d', 'WideBatchNorm2d', 'WideLayerNorm',
    'WideGroupNorm', 'GroupNormStrategy',
    'WideInstanceNorm1d', 'WideInstanceNorm2d', 'InstanceNormStrategy',
    'WideEmbedding', 'EmbeddingStrategy',
    'WideAttention', 'AttentionStrategy',
    'WideGRU', 'GRUStrategy',
    'WideLSTM', 'LSTMStrategy',
    'BUILTIN_PRIMITIVES',
]
