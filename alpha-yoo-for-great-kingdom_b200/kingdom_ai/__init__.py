"""B200-native batched self-play for the 9x9 Great Kingdom game.

Drop-in for the GPU self-play path of ``kingdom_ai`` (GpuStateBatch, GpuPUCT,
GpuPUCTOptions, GpuSearchResult, collect_gpu_puct_games). All kernels live in
``libgk.so`` (CUDA for sm_100a) behind the C ABI of ``include/gk.h``.
"""

from .gpu_rules import (  # noqa: F401
    GPU_ACTION_SIZE, GPU_ACTOR, GPU_BLACK_STOCK, GPU_CAPTURE, GPU_CAPTURED, GPU_CELL_COUNT, GPU_NONE,
    GPU_PASSES, GPU_REASON, GPU_RESERVED, GPU_STATE_WIDTH, GPU_SUICIDE, GPU_TWO_PASSES, GPU_WHITE_STOCK,
    GPU_WINNER, GpuStateBatch,
)
from .gpu_puct import GpuPUCT, GpuPUCTOptions, GpuSearchResult, HashEvaluator  # noqa: F401
from .training import Cell, EndReason, GameData, TrainingBatch, TrainingSample, collect_gpu_puct_games  # noqa: F401
from .replay import DeviceReplayBuffer, validate_rows  # noqa: F401
from .batched_puct import BatchedSearchResult, GpuBatchedPUCT, PUCTOptions  # noqa: F401
from .evaluation import EvaluationResult, evaluate_models_gpu  # noqa: F401
from .engine_api import BatchedPUCT, PUCTMoveStatistics, PUCTSearchResult, encode_puct_batch  # noqa: F401
