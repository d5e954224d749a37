# Build, test and benchmark entry points (the reference exposes its tests as `make test*`).
#
#   make build            compile the sm_100a extension in-tree
#   make test             CPU suite: units + multi-rank gloo (TP/SP, ZeRO-0..3, PP, resume, failures)
#   make test-unit        pure unit tests only (incl. benchmark configurations, clock sampler)
#   make test-race        model check of the cross-GPU flag protocols (random interleavings)
#   make test-integration multi-rank CPU tests and the CLI
#   make test-quick       unit tests + the 2-rank ZeRO stage and TP equivalence checks
#   make test-gpu         kernels, model and bounded-wait tests on a B200 (pytest -m gpu)
#   make bench            headline benchmark on GPUS GPUs (default 1)
#   make train-tiny       tiny LLaMA, TP=2, ZeRO-3 on two CPU gloo ranks
#
# TIMEOUT bounds each pytest invocation (seconds).

PYTHON ?= python
GPUS ?= 1
TIMEOUT ?= 1800
PORT ?= 29511

.PHONY: build test test-unit test-race test-integration test-quick test-gpu bench train-tiny clean

build:
	$(PYTHON) setup.py build_ext --inplace

test:
	timeout $(TIMEOUT) $(PYTHON) -m pytest tests -q -m "not gpu"

test-unit:
	timeout $(TIMEOUT) $(PYTHON) -m pytest tests/test_units.py tests/test_model_vs_hf.py \
		tests/test_bench_config.py tests/test_clocks.py -q

test-race:
	timeout $(TIMEOUT) $(PYTHON) -m pytest tests/test_protocol_model.py -q

test-integration:
	timeout $(TIMEOUT) $(PYTHON) -m pytest tests/test_distributed_cpu.py tests/test_cli.py -q

test-quick:
	timeout $(TIMEOUT) $(PYTHON) -m pytest tests/test_units.py -q
	timeout $(TIMEOUT) $(PYTHON) -m pytest tests/test_distributed_cpu.py -q -k "zero_stages_agree or tp_model_matches"

test-gpu:
	timeout $(TIMEOUT) $(PYTHON) -m pytest tests -q -m gpu

bench:
ifeq ($(GPUS),1)
	$(PYTHON) bench.py
else
	$(PYTHON) -m torch.distributed.run --nnodes=1 --nproc-per-node $(GPUS) --master-addr 127.0.0.1 \
		--master-port $(PORT) bench.py --gpus $(GPUS)
endif

train-tiny:
	CUDA_VISIBLE_DEVICES= $(PYTHON) -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 \
		--master-port $(PORT) -m femtotron_b200.scripts.train --config configs/tiny_llama_debug.yaml \
		--tp 2 --zero_stage 3 --train_steps 10 --checkpoint_dir /tmp/femtotron_b200_ckpt

clean:
	rm -rf build femtotron_b200/_C*.so
