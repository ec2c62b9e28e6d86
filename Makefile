# Build the sm_100a extension in place, test, benchmark.
.PHONY: build test test-gpu test-all data train bench bench-ref thesis profile validate lint clean

PY ?= python
NGPU ?= 1

build:
	$(PY) setup.py build_ext --inplace

test:
	$(PY) -m pytest tests -m "not gpu"

test-gpu: build
	$(PY) -m pytest tests -m gpu

test-all: build
	$(PY) -m pytest tests

data:
	$(PY) -m packbalance_b200.data.prepare --config configs/tiny.yaml

train:
	$(PY) -m torch.distributed.run --standalone --local-addr 127.0.0.1 --nproc-per-node $(NGPU) \
		-m packbalance_b200.train.train --config configs/tiny.yaml

bench: build
	if [ "$(NGPU)" = "1" ]; then $(PY) bench.py; else \
	$(PY) -m torch.distributed.run --nnodes=1 --nproc-per-node $(NGPU) --master-addr 127.0.0.1 \
		--master-port 29531 bench.py --gpus $(NGPU); fi

bench-ref:
	$(PY) bench.py --impl reference

thesis:
	$(PY) -m packbalance_b200.profiling.prove_intuition --config configs/bench.yaml

profile:
	$(PY) -m packbalance_b200.train.train --config configs/tiny.yaml --profile

validate: build
	bash packbalance_b200/profiling/gpu_validate.sh

lint:
	ruff check .

clean:
	rm -rf build artifacts .pytest_cache .ruff_cache packbalance_b200/*.so
