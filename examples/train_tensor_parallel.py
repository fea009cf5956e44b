"""Tensor parallelism example.

Run, e.g.: `torchrun --standalone --local-addr 127.0.0.1 --nproc-per-node N examples/train_tensor_parallel.py --config configs/tensor_parallel_2gpu.yaml`
"""

from _common import run_training

if __name__ == "__main__":
    run_training("Tensor parallelism", "tensor_parallel_2gpu.yaml")
