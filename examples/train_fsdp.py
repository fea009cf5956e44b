"""Flat-parameter FSDP example.

Run, e.g.: `torchrun --standalone --local-addr 127.0.0.1 --nproc-per-node N examples/train_fsdp.py --config configs/fsdp_4gpu.yaml`
"""

from _common import run_training

if __name__ == "__main__":
    run_training("Flat-parameter FSDP", "fsdp_4gpu.yaml")
