"""Bucketed DDP example.

Run, e.g.: `torchrun --standalone --local-addr 127.0.0.1 --nproc-per-node N examples/train_ddp.py --config configs/ddp_2gpu.yaml`
"""

from _common import run_training

if __name__ == "__main__":
    run_training("Bucketed DDP", "ddp_2gpu.yaml")
