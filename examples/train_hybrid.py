"""Full 4-D hybrid grid example.

Run, e.g.: `torchrun --standalone --local-addr 127.0.0.1 --nproc-per-node N examples/train_hybrid.py --config configs/hybrid_8gpu.yaml`
"""

from _common import run_training

if __name__ == "__main__":
    run_training("Full 4-D hybrid grid", "hybrid_8gpu.yaml")
