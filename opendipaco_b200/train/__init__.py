from .loop import (
    DiPaCoEngine, ExecOptions, RoundMetrics, batch_indices, config_fingerprint, run_inner_steps,
    token_loss_sum,
)
from .memory import fits, fused_breakdown, measure_peak, vram_breakdown

__all__ = ["DiPaCoEngine", "ExecOptions", "RoundMetrics", "batch_indices", "config_fingerprint",
           "run_inner_steps", "token_loss_sum", "fits", "fused_breakdown", "measure_peak",
           "vram_breakdown"]
