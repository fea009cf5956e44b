"""Megatron sequence parallelism example.

Run, e.g.: `torchrun --standalone --local-addr 127.0.0.1 --nproc-per-node N examples/train_sequence_parallel.py --config configs/sequence_parallel_2gpu.yaml`
"""

from _common import run_training

if __name__ == "__main__":
    run_training("Megatron sequence parallelism", "sequence_parallel_2gpu.yaml")
