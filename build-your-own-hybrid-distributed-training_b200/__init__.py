"""hybrid_training -- a B200-native hybrid-parallel training framework.

Strategies: bucketed DDP (:mod:`.parallel.ddp`), flat-parameter FSDP and
hybrid sharding (:mod:`.parallel.fsdp`), tensor parallelism
(:mod:`.parallel.tensor_parallel`), sequence parallelism
(:mod:`.parallel.sequence_parallel`), their composition over a 4-D rank grid
(:mod:`.parallel.hybrid`), and manifest-based resharding checkpoints
(:mod:`.checkpoint`).  Hot operations run as hand-written sm_100a kernels
(:mod:`.ops`), including collectives fused with their GEMMs over NVLink peer
memory.  The public API matches ``build-your-own-hybrid-distributed-training``
(``src/hybrid_training/__init__.py:18-32``).
"""

from .config import ExperimentConfig, TopologyConfig, load_experiment_config
from .errors import HybridTrainingError
from .logging import configure_logging, get_logger

__version__ = "0.1.0"

__all__ = [
    "ExperimentConfig",
    "HybridTrainingError",
    "TopologyConfig",
    "__version__",
    "configure_logging",
    "get_logger",
    "load_experiment_config",
]
