from .adam8bit import Adam8bit
from .diloco import (
    apply_outer_grads, inner_lr_at, make_inner_optimizer, make_outer_optimizer, module_delta,
)

__all__ = ["Adam8bit", "apply_outer_grads", "inner_lr_at", "make_inner_optimizer",
           "make_outer_optimizer", "module_delta"]
