# Developer commands.  `make help` lists them; PROFILE selects a pipeline profile (a built-in name or a
# directory holding model.yaml / data.yaml / training.yaml).
PYTHON ?= python
PROFILE ?= cpu_smoke
NGPU ?= 1

.PHONY: help build validate smoke profiles check test test-gpu test-config test-inference test-training test-distributed bench

help: ## Show the available commands.
	@grep -E "^[a-z-]+:.*## " $(MAKEFILE_LIST) | sed -e "s/:.*## /\t/"

build: ## Compile the sm_100a CUDA extension in-tree (kimi_k3_b200/_C*.so).
	$(PYTHON) -c "import __graft_entry__ as g; g.build()"

validate: ## Validate PROFILE (configs and their compatibility) without building a model.
	$(PYTHON) -m kimi_k3_b200 train --profile $(PROFILE) --validate-only

smoke: ## Train the tiny model for a few steps on CPU, then decode 8 tokens.
	$(PYTHON) -m kimi_k3_b200 smoke

profiles: ## Write every built-in pipeline profile under configs/kimi_full_pipeline.
	$(PYTHON) -m kimi_k3_b200 profiles

check: ## Fast contract checks: configs, CLI, import map, primitives.
	$(PYTHON) -m pytest -q tests/test_config_cpu.py tests/test_api_map_cpu.py tests/test_primitives_cpu.py

test: ## The whole CPU suite (float64 oracles, gloo multi-process layouts).
	$(PYTHON) -m pytest -q -m "not gpu" tests

test-gpu: ## Kernel numerics and GPU paths (needs a B200 and the built extension).
	$(PYTHON) -m pytest -q -m gpu tests

test-config: ## Every pipeline profile and the CLI.
	$(PYTHON) -m pytest -q tests/test_config_cpu.py

test-inference: ## Sampling, checkpoint loading, cached and graph decode, sharded decode.
	$(PYTHON) -m pytest -q -m "not gpu" tests/test_inference_cpu.py tests/test_infer_session_cpu.py tests/test_distributed_infer_cpu.py

test-training: ## Optimizers, schedules, curriculum, diagnostics, checkpoints and the trainer.
	$(PYTHON) -m pytest -q -m "not gpu" tests/test_optimizer_cpu.py tests/test_optimizer_rules_cpu.py tests/test_legacy_optimizers_cpu.py tests/test_training_rules_cpu.py tests/test_training_services_cpu.py tests/test_curriculum_cpu.py tests/test_diagnostics_cpu.py tests/test_trainer_cpu.py

test-distributed: ## DP / TP / EP / FSDP layouts, checkpoints and runtime rules on gloo ranks.
	$(PYTHON) -m pytest -q -m "not gpu" tests/test_distributed_cpu.py tests/test_distributed_rules_cpu.py tests/test_distributed_infer_cpu.py

bench: ## The flagship training-step benchmark on NGPU GPUs of this node.
	@if [ "$(NGPU)" = "1" ]; then $(PYTHON) bench.py; else \
	$(PYTHON) -m torch.distributed.run --nnodes=1 --nproc-per-node $(NGPU) --master-addr 127.0.0.1 bench.py --gpus $(NGPU); fi
