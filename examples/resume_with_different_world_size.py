"""Resume a checkpoint at a different data-parallel / shard width (the tensor width must match).

Save with N ranks (e.g. the FSDP-4 config), then run this with M ranks:
`torchrun --standalone --local-addr 127.0.0.1 --nproc-per-node 2 examples/resume_with_different_world_size.py
 --config configs/fsdp_2gpu.yaml --resume <checkpoint-dir>`.  The global batch is kept constant by scaling the
micro-batch, so the resumed loss curve continues the original one.
"""

import dataclasses

from _common import load_config, parser, report_environment, report_result

from hybrid_training.checkpoint import read_metadata
from hybrid_training.distributed import distributed_context
from hybrid_training.training import TrainingEngine

if __name__ == "__main__":
    p = parser("resume at a different world size", "fsdp_2gpu.yaml")
    p.add_argument("--resume", required=True, help="checkpoint directory to resume from")
    args = p.parse_args()
    cfg = load_config(args)
    meta = read_metadata(args.resume)
    saved = meta.get("config") or {}
    saved_global = saved.get("data", {}).get("micro_batch_size", cfg.data.micro_batch_size) * meta.get("world_size", 1)
    with distributed_context(cfg) as ctx:
        data_ranks = ctx.group("dp_shard").size
        if saved_global % data_ranks == 0:
            cfg = dataclasses.replace(cfg, data=dataclasses.replace(cfg.data, micro_batch_size=saved_global // data_ranks))
        report_environment(ctx, show_topology=args.show_topology)
        engine = TrainingEngine(cfg, ctx)
        loaded = engine.load_checkpoint(args.resume)
        if ctx.is_primary:
            print(f"resumed {loaded}")
        engine.train()
        report_result(ctx, engine)
        engine.close()
