from .trainer import Trainer

__all__ = ["Trainer"]
from .checkpoint import load_checkpoint, load_sharded, save_checkpoint, save_sharded  # noqa: E402

__all__ += ["save_checkpoint", "load_checkpoint", "save_sharded", "load_sharded"]
