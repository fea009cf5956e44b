# Developer entry points.  Every GPU target expects one process per GPU on one node.
PYTHON ?= python
NPROC ?= 2
PORT ?= 29511
TORCHRUN = $(PYTHON) -m torch.distributed.run --nnodes=1 --nproc-per-node $(NPROC) --master-addr 127.0.0.1 --master-port $(PORT)

.PHONY: help build test test-unit test-distributed test-gpu test-multigpu bench bench-reference bench-scaling \
        examples-cpu example-hybrid inspect clean

help:
	@echo "build            compile the sm_100a extension in-tree (ops/_C*.so)"
	@echo "test             CPU suite (unit, Gloo multi-process, checkpoint, source rules)"
	@echo "test-unit        single-process CPU tests only"
	@echo "test-distributed Gloo multi-process tests only"
	@echo "test-gpu         GPU tests (B200); multi-GPU tests run when >= 2 GPUs are visible"
	@echo "bench            headline benchmark on NPROC GPUs (GPT-2-124M DDP); CONFIG=llama_fsdp|llama_tp_sp|llama_hybrid"
	@echo "bench-reference  the reference implementation on the same config"
	@echo "bench-scaling    headline benchmark at 1, 2, 4 and 8 GPUs"
	@echo "examples-cpu     every example on 2 CPU ranks (Gloo)"
	@echo "example-hybrid   the 4-D hybrid example on NPROC GPUs"
	@echo "inspect CKPT=... print a checkpoint's manifest summary and reshard plan"

build:
	$(PYTHON) -c "import __graft_entry__ as g; g.build()"

test:
	$(PYTHON) -m pytest tests -q -m "not gpu"

test-unit:
	$(PYTHON) -m pytest tests -q -m "not gpu and not distributed"

test-distributed:
	$(PYTHON) -m pytest tests -q -m "distributed and not gpu"

test-gpu:
	NCCL_NVLS_ENABLE=0 $(PYTHON) -m pytest tests -q -m gpu

test-multigpu:
	NCCL_NVLS_ENABLE=0 $(PYTHON) -m pytest tests -q -m multigpu

CONFIG ?= gpt2_ddp
STEPS ?= 20
WARMUP ?= 5
bench:
ifeq ($(NPROC),1)
	$(PYTHON) bench.py --gpus 1 --steps $(STEPS) --warmup $(WARMUP) --config $(CONFIG)
else
	$(TORCHRUN) bench.py --gpus $(NPROC) --steps $(STEPS) --warmup $(WARMUP) --config $(CONFIG)
endif

bench-reference:
ifeq ($(NPROC),1)
	$(PYTHON) bench.py --impl reference --gpus 1 --steps $(STEPS) --warmup $(WARMUP)
else
	$(TORCHRUN) bench.py --impl reference --gpus $(NPROC) --steps $(STEPS) --warmup $(WARMUP)
endif

bench-scaling:
	$(PYTHON) bench.py --gpus 1 --steps $(STEPS) --warmup $(WARMUP)
	for n in 2 4 8; do \
	  $(PYTHON) -m torch.distributed.run --nnodes=1 --nproc-per-node $$n --master-addr 127.0.0.1 --master-port $(PORT) \
	    bench.py --gpus $$n --steps $(STEPS) --warmup $(WARMUP) || exit 1; \
	done

examples-cpu:
	for pair in train_ddp:ddp_2gpu train_fsdp:fsdp_2gpu train_tensor_parallel:tensor_parallel_2gpu \
	            train_sequence_parallel:sequence_parallel_2gpu; do \
	  ex=$${pair%%:*}; cfg=$${pair##*:}; \
	  $(PYTHON) -m torch.distributed.run --nnodes=1 --nproc-per-node 2 --master-addr 127.0.0.1 --master-port $(PORT) \
	    examples/$$ex.py --config configs/$$cfg.yaml --backend gloo --device cpu --steps 2 || exit 1; \
	done

example-hybrid:
	$(TORCHRUN) examples/train_hybrid.py --config configs/hybrid_8gpu.yaml

inspect:
	$(PYTHON) -m hybrid_training.checkpoint.reader $(CKPT) --plan

clean:
	rm -rf build-your-own-hybrid-distributed-training_b200/ops/_build .pytest_cache
