"""GPT-2-124M-shape DDP on B200 (bf16, CUDA graph) example.

Run, e.g.: `torchrun --standalone --local-addr 127.0.0.1 --nproc-per-node N examples/train_gpt2_124m.py --config configs/gpt2_124m_ddp_8gpu.yaml`
"""

from _common import run_training

if __name__ == "__main__":
    run_training("GPT-2-124M-shape DDP on B200 (bf16, CUDA graph)", "gpt2_124m_ddp_8gpu.yaml")
