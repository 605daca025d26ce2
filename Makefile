# SPDX-License-Identifier: Apache-2.0
# Builds libvccl.so (sm_100a) plus the native tools and tests into
# vkccl_b200/_native/.  `make -j` from the repository root.

CUDA_HOME ?= /usr/local/cuda
NVCC      ?= $(CUDA_HOME)/bin/nvcc
ARCH      ?= -gencode arch=compute_100a,code=sm_100a
OUT       := vkccl_b200/_native
OBJ       := $(OUT)/obj
BIN       := $(OUT)/bin

NVFLAGS := $(ARCH) -O3 -lineinfo -std=c++17 -Xcompiler -fPIC -Xcompiler -Wall \
           -Iinclude -Icsrc -I$(CUDA_HOME)/include --expt-relaxed-constexpr \
           -diag-suppress 177,550,20281
LDFLAGS := -cudart static -lpthread -ldl -lrt

LIB_CC  := $(wildcard csrc/common/*.cc csrc/control/*.cc csrc/runtime/*.cc)
LIB_CU  := $(wildcard csrc/runtime/*.cu csrc/fused/*.cu)
LIB_OBJ := $(patsubst csrc/%,$(OBJ)/%.o,$(LIB_CC) $(LIB_CU))
HDRS    := $(wildcard include/*.h csrc/*/*.h csrc/*/*.cuh)

TOOLS   := $(BIN)/vccl-bench $(BIN)/vccl-info $(BIN)/vccl-devbuf-demo $(BIN)/vccl-barrier-bench
TESTS   := $(BIN)/test_bootstrap $(BIN)/test_collectives $(BIN)/test_control $(BIN)/test_tiling $(BIN)/test_tuning \
           $(BIN)/test_coll_index $(BIN)/test_dmabuf $(BIN)/test_regcache

all: $(OUT)/libvccl.so $(TOOLS) $(TESTS)

$(OBJ)/%.cc.o: csrc/%.cc $(HDRS)
	@mkdir -p $(dir $@)
	$(NVCC) $(NVFLAGS) -x cu -c $< -o $@

$(OBJ)/%.cu.o: csrc/%.cu $(HDRS)
	@mkdir -p $(dir $@)
	$(NVCC) $(NVFLAGS) -c $< -o $@

$(OUT)/libvccl.so: $(LIB_OBJ)
	$(NVCC) $(ARCH) -shared -o $@ $^ $(LDFLAGS)

$(BIN)/%: csrc/tools/%.cc $(OUT)/libvccl.so include/vccl.h
	@mkdir -p $(BIN)
	$(NVCC) $(NVFLAGS) -x cu $< -o $@ -L$(OUT) -lvccl -Xlinker -rpath,'$$ORIGIN/..' $(LDFLAGS)

$(BIN)/test_%: csrc/tests/test_%.cc $(OUT)/libvccl.so $(HDRS)
	@mkdir -p $(BIN)
	$(NVCC) $(NVFLAGS) -x cu $< -o $@ -L$(OUT) -lvccl -Xlinker -rpath,'$$ORIGIN/..' $(LDFLAGS)

clean:
	rm -rf $(OUT)/obj $(OUT)/bin $(OUT)/libvccl.so $(OUT)/kit $(KIT_TAR)

# Bring-up kit (the counterpart of the reference's kit/build-kit.sh): the library, the
# tools, the native collective and dmabuf tests, the headers and the
# bring-up script in one tarball that runs on any node with a CUDA driver
# (the CUDA runtime is linked statically; binaries find libvccl.so through
# their $$ORIGIN/.. rpath).  `make kit` -> vkccl_b200/_native/vccl-e2e-kit-<arch>.tar.gz
KIT     := $(OUT)/kit
KIT_TAR := $(OUT)/vccl-e2e-kit-$(shell uname -m).tar.gz

kit: $(KIT_TAR)

$(KIT_TAR): $(OUT)/libvccl.so $(TOOLS) $(BIN)/test_collectives $(BIN)/test_dmabuf csrc/tools/vccl-e2e.sh
	rm -rf $(KIT)
	mkdir -p $(KIT)/bin $(KIT)/include
	cp $(OUT)/libvccl.so $(KIT)/
	cp $(TOOLS) $(BIN)/test_collectives $(BIN)/test_dmabuf csrc/tools/vccl-e2e.sh $(KIT)/bin/
	cp include/*.h $(KIT)/include/
	tar -C $(OUT) -czf $@ kit

.PHONY: all clean kit

# Host-only control plane and host data plane (no CUDA runtime) built with
# sanitizers for the CPU race checks: `make sanitize` ->
# bin/test_{bootstrap,hostplane}_threads_{tsan,asan}.
CTRL_SRC := csrc/common/types.cc csrc/common/env.cc csrc/common/log.cc csrc/common/net.cc csrc/control/bootstrap.cc
SAN_FLAGS := -std=c++17 -O1 -g -Iinclude -Icsrc -pthread

$(BIN)/test_bootstrap_threads_tsan: csrc/tests/test_bootstrap_threads.cc $(CTRL_SRC) $(HDRS)
	@mkdir -p $(BIN)
	g++ $(SAN_FLAGS) -fsanitize=thread csrc/tests/test_bootstrap_threads.cc $(CTRL_SRC) -o $@

$(BIN)/test_bootstrap_threads_asan: csrc/tests/test_bootstrap_threads.cc $(CTRL_SRC) $(HDRS)
	@mkdir -p $(BIN)
	g++ $(SAN_FLAGS) -fsanitize=address,undefined csrc/tests/test_bootstrap_threads.cc $(CTRL_SRC) -o $@

# The host data plane (TCP mesh, sender thread) on top of it; its element
# types come from the CUDA headers, which compile as host code.
HP_SRC := csrc/runtime/hostplane.cc $(CTRL_SRC)

$(BIN)/test_hostplane_threads_tsan: csrc/tests/test_hostplane_threads.cc $(HP_SRC) $(HDRS)
	@mkdir -p $(BIN)
	g++ $(SAN_FLAGS) -I$(CUDA_HOME)/include -fsanitize=thread csrc/tests/test_hostplane_threads.cc $(HP_SRC) -o $@

$(BIN)/test_hostplane_threads_asan: csrc/tests/test_hostplane_threads.cc $(HP_SRC) $(HDRS)
	@mkdir -p $(BIN)
	g++ $(SAN_FLAGS) -I$(CUDA_HOME)/include -fsanitize=address,undefined csrc/tests/test_hostplane_threads.cc $(HP_SRC) -o $@

sanitize: $(BIN)/test_bootstrap_threads_tsan $(BIN)/test_bootstrap_threads_asan \
          $(BIN)/test_hostplane_threads_tsan $(BIN)/test_hostplane_threads_asan

.PHONY: sanitize

# The reference's own build for `bench.py --impl reference` (TCP only, from an
# unmodified copy of its source): make reference REF_SRC=<reference checkout>.
# Output: baseline/_ref/build/libvccl.so (+ its tools and tests) and
# baseline/_ref/vccl (its Python package); git-ignored, carried to GPU boxes.
reference:
	@test -n "$(REF_SRC)" || (echo "usage: make reference REF_SRC=<reference checkout>"; exit 1)
	rm -rf _build/refsrc && mkdir -p _build/refsrc baseline/_ref
	cp -r $(REF_SRC)/. _build/refsrc/
	cmake -S _build/refsrc -B baseline/_ref/build -DVCCL_ENABLE_VERBS=OFF -DCMAKE_BUILD_TYPE=Release
	cmake --build baseline/_ref/build -j8
	rm -rf baseline/_ref/vccl && cp -r _build/refsrc/python/vccl baseline/_ref/vccl

.PHONY: reference
