from .model import get_compiled_to_uncompiled_mapping, get_model_params
from .profile import GPU_PEAK_FLOPS, compute_mfu, get_gpu_peak_flops, measured_peak_flops
from .training import get_training_info, set_seed

__all__ = ["get_training_info", "set_seed", "get_model_params", "get_compiled_to_uncompiled_mapping",
           "get_gpu_peak_flops", "compute_mfu", "GPU_PEAK_FLOPS", "measured_peak_flops"]
