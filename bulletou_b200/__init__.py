"""bulletou_b200 -- B200-native (sm_100a) implementation of BulletOu's training hot path.

The compute lives in libbulletou_b200.so (hand-written CUDA behind a C ABI that
mirrors the reference's cuda-cpp backend); this package is the host-side
mirror of the reference's Rust crate API (see cuda_cpp.py) plus the seeded
synthetic data generator used by tests and benchmarks.
"""
from ._lib import CudaCppError, Library, library, reference_library  # noqa: F401
from .cuda_cpp import (  # noqa: F401
    FLT_MAX,
    NNUE_HALFKP_256X2_32_32,
    Context,
    Event,
    F32Buffer,
    GraphExec,
    I32Buffer,
    KpptTableTrainStepRunner,
    NnueForwardHostWeights,
    NnueForwardShape,
    NnueTrainStepHostBatch,
    NnueTrainStepRunner,
    RAdamUpdateParams,
    RangerUpdateParams,
    ScalarLossKind,
    nnue_forward_host,
    ranger_update_device,
    ranger_update_host,
    ranger_update_stacked_dirty_device,
    scalar_loss_host,
)

from .sfnn import (  # noqa: F401
    SFNN_HALFKA_HM2_1536_15_32_K3K3,
    QuantizedRounding,
    QuantizedSfnnDeviceWeights,
    SfnnIntegerForwardWorkspace,
    SfnnLayerLrMultipliers,
    SfnnFactorizerAlpha,
    SfnnForwardHostWeights,
    SfnnForwardShape,
    SfnnTrainStepHostBatch,
    SfnnTrainStepRunner,
    sfnn_backward_device,
    sfnn_backward_train_profile_device,
    sfnn_build_quantized_proxy_device,
    sfnn_integer_forward_device,
    sfnn_quantize_device,
)

from .nnue_quant import (  # noqa: F401
    NnueIntegerForwardWorkspace,
    QuantizedNnueDeviceWeights,
    nnue_integer_forward_device,
    nnue_quantize_device,
)

from .teacher import (  # noqa: F401
    PSV_DTYPE,
    LayerStackBucketKind,
    TeacherBatch,
    TeacherBatchConfig,
    TeacherBatchProducer,
    TeacherUploadSlot,
    WinRateModelTargetParams,
    teacher_prepare_device,
    win_rate_model_score_table,
)

from .validate import AccuracyReport, ValidationLossKind, ValidationMetrics, sfnn_validation_stats  # noqa: F401
from .nn_bin import (  # noqa: F401
    nnue_nn_bin_bytes, parse_nnue_nn_bin, parse_sfnn_nn_bin, read_nnue_nn_bin, read_sfnn_nn_bin, sfnn_nn_bin_bytes,
    write_nnue_nn_bin, write_sfnn_nn_bin,
)

from .state_bin import (  # noqa: F401
    CheckpointLog, SfnnTrainState, latest_complete_checkpoint_dir, load_halfkp_state, load_sfnn_state,
    parse_model_weights_bin, restore_halfkp_runner, restore_sfnn_runner, write_checkpoint_dir, write_halfkp_checkpoint,
    write_halfkp_state_bin, write_sfnn_checkpoint, write_sfnn_state_bin,
)
from .revive import (  # noqa: F401
    Contribution, FtCalibration, L1Calibration, L2Calibration, begin_revival_epoch, compensate_ft_revival_mean,
    compensate_l1_revival_mean, revive_ft, revive_ft_units, revive_l1_selected, revive_l2, revive_l2_selected,
    saturated_units,
)

__version__ = "0.1.0"
