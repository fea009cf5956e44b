"""Train a few steps, save a checkpoint, and print its inspection summary.

Run: `torchrun --standalone --local-addr 127.0.0.1 --nproc-per-node 4 examples/save_distributed_checkpoint.py`
"""

import json

from _common import load_config, parser, report_environment

from hybrid_training.checkpoint import inspect_checkpoint
from hybrid_training.distributed import distributed_context
from hybrid_training.training import TrainingEngine

if __name__ == "__main__":
    args = parser("save a distributed checkpoint", "fsdp_4gpu.yaml").parse_args()
    cfg = load_config(args)
    with distributed_context(cfg) as ctx:
        report_environment(ctx, show_topology=args.show_topology)
        engine = TrainingEngine(cfg, ctx)
        engine.train()
        path = engine.save_checkpoint()
        if ctx.is_primary:
            print(json.dumps(inspect_checkpoint(path), indent=2, sort_keys=True))
        engine.close()
