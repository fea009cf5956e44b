"""Llama-shaped FSDP / TP+SP on B200 example.

Run, e.g.: `torchrun --standalone --local-addr 127.0.0.1 --nproc-per-node N examples/train_llama.py --config configs/llama_1b3_fsdp_8gpu.yaml`
"""

from _common import run_training

if __name__ == "__main__":
    run_training("Llama-shaped FSDP / TP+SP on B200", "llama_1b3_fsdp_8gpu.yaml")
