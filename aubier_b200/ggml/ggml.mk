# ggml.mk -- builds the ggml side of the drop-in boundary against the reference's vendored ggml.
#
# The reference's tree (llama.cpp @ 50e3e3e4, vendor/llama.cpp/ggml/) already carries its M4 patch
# (patches/ggml-m4/custom-op-m4.patch).  This recipe copies ggml's include/ and src/ into a build
# folder, applies m4b-ggml.patch there (builders for both head geometries and the ragged KQKV,
# ggml-cuda's dispatch include and supports_op through libm4b), adds the ggml-cuda shim
# (m4-b200.cu/.cuh), and then
#   - compiles the patched ggml-cuda.cu and the shim with nvcc for sm_100a (the backend's dispatch
#     and supports_op hooks and the launchers, against ggml-cuda's own headers);
#   - builds the patched ggml core + ggml-cpu with gcc/g++ and links m4b_ggml_check, which builds
#     the M4 nodes through ggml's builders and asks libm4b's supports_op (tests/test_ggml_boundary.py);
#   - compiles the engine's layer graph (engine/m1_layer.cpp) with m1-layer-batch.patch, which
#     keeps the fused ops for token batches (KQKV over each row's window).
# The reference's CMake is not run: the source lists and definitions below are this file's own.
# Every output goes to $(OUT), which is git-ignored and not sent to the GPU box.
#
# usage: make -f aubier_b200/ggml/ggml.mk REF=<reference root> OUT=aubier_b200/ggml/_build -j8

REF ?= /nonexistent
OUT ?= aubier_b200/ggml/_build
HERE := aubier_b200/ggml
GG   := $(REF)/vendor/llama.cpp/ggml
TREE := $(OUT)/ggml
NVCC ?= nvcc

BASE_C   := ggml.c ggml-alloc.c ggml-quants.c
BASE_CXX := ggml.cpp ggml-backend.cpp ggml-backend-meta.cpp ggml-opt.cpp ggml-threading.cpp gguf.cpp
CPU_C    := ggml-cpu/ggml-cpu.c ggml-cpu/quants.c ggml-cpu/arch/x86/quants.c
CPU_CXX  := ggml-cpu/ggml-cpu.cpp ggml-cpu/repack.cpp ggml-cpu/hbm.cpp ggml-cpu/traits.cpp \
            ggml-cpu/amx/amx.cpp ggml-cpu/amx/mmq.cpp ggml-cpu/binary-ops.cpp \
            ggml-cpu/unary-ops.cpp ggml-cpu/vec.cpp ggml-cpu/ops.cpp \
            ggml-cpu/tiled/tiled.cpp ggml-cpu/tiled/tiled-kernel.cpp \
            ggml-cpu/llamafile/sgemm.cpp ggml-cpu/arch/x86/repack.cpp

DEFS   := -DNDEBUG -D_GNU_SOURCE -D_XOPEN_SOURCE=600 -DGGML_USE_LLAMAFILE -DGGML_USE_CPU \
          -DGGML_SCHED_MAX_COPIES=4
INCS   := -I$(OUT)/gen -I$(TREE)/include -I$(TREE)/src -I$(TREE)/src/ggml-cpu
COMMON := -O2 -fPIC -pthread -march=x86-64-v3 $(DEFS) $(INCS) -Wno-unused-result
CUDA_FLAGS := -std=c++17 -gencode arch=compute_100a,code=sm_100a -O2 -Xcompiler -fPIC \
              -DGGML_USE_CUDA -DGGML_CUDA_USE_GRAPHS -I$(OUT)/gen -I$(TREE)/include \
              -I$(TREE)/src -I$(TREE)/src/ggml-cuda -Iinclude

OBJS := $(addprefix $(OUT)/obj/,$(addsuffix .o,$(BASE_C) $(BASE_CXX) $(CPU_C) $(CPU_CXX)))

all: $(OUT)/m4b_ggml_check $(OUT)/cuda/ggml-cuda.o $(OUT)/cuda/m4-b200.o $(OUT)/engine/m1_layer.o

$(OUT)/gen/ggml-version.h:
	@mkdir -p $(dir $@)
	@printf '#pragma once\n#define GGML_VERSION "0.26.0"\n#define GGML_COMMIT "50e3e3e4"\n' > $@

# the patched tree; rebuilt when the patch or the shim changes
$(OUT)/.patched: $(HERE)/m4b-ggml.patch $(HERE)/m4-b200.cu $(HERE)/m4-b200.cuh
	@test -d $(GG)/src || { echo "reference ggml not found under $(GG)"; exit 1; }
	rm -rf $(TREE) $(OUT)/obj $(OUT)/cuda
	mkdir -p $(TREE)
	cp -r $(GG)/include $(GG)/src $(TREE)/
	patch -s -d $(TREE) -p1 < $(HERE)/m4b-ggml.patch
	cp $(HERE)/m4-b200.cu $(HERE)/m4-b200.cuh $(TREE)/src/ggml-cuda/
	touch $@

$(TREE)/src/%: $(OUT)/.patched ;

$(OUT)/obj/%.c.o: $(OUT)/.patched $(OUT)/gen/ggml-version.h
	@mkdir -p $(dir $@)
	gcc -std=gnu11 $(COMMON) -c $(TREE)/src/$*.c -o $@

$(OUT)/obj/%.cpp.o: $(OUT)/.patched $(OUT)/gen/ggml-version.h
	@mkdir -p $(dir $@)
	g++ -std=gnu++17 $(COMMON) -c $(TREE)/src/$*.cpp -o $@

$(OUT)/obj/m4b_ggml_check.o: $(HERE)/m4b_ggml_check.c $(OUT)/.patched $(OUT)/gen/ggml-version.h
	@mkdir -p $(dir $@)
	gcc -std=gnu11 $(COMMON) -Iinclude -c $< -o $@

$(OUT)/m4b_ggml_check: $(OBJS) $(OUT)/obj/m4b_ggml_check.o aubier_b200/libm4b.so
	g++ -pthread -o $@ $(OBJS) $(OUT)/obj/m4b_ggml_check.o -Laubier_b200 -lm4b \
	    -Wl,-rpath,$(abspath aubier_b200) -lm

$(OUT)/cuda/ggml-cuda.o: $(OUT)/.patched $(OUT)/gen/ggml-version.h
	@mkdir -p $(dir $@)
	$(NVCC) $(CUDA_FLAGS) -c $(TREE)/src/ggml-cuda/ggml-cuda.cu -o $@

$(OUT)/cuda/m4-b200.o: $(OUT)/.patched $(OUT)/gen/ggml-version.h include/m4b.h
	@mkdir -p $(dir $@)
	$(NVCC) $(CUDA_FLAGS) -c $(TREE)/src/ggml-cuda/m4-b200.cu -o $@

# the engine's layer graph with m1-layer-batch.patch (the fused ops kept at nt > 1, KQKV over the
# rows' windows), compiled against the patched ggml headers: the caller side of the ragged path
ENGINE_SRC := m1_layer.cpp m1_layer.h gguf_model.h store.h
$(OUT)/engine/.patched: $(HERE)/m1-layer-batch.patch
	@test -d $(REF)/engine || { echo "reference engine not found under $(REF)"; exit 1; }
	rm -rf $(OUT)/engine && mkdir -p $(OUT)/engine
	cp $(addprefix $(REF)/engine/,$(ENGINE_SRC)) $(OUT)/engine/
	patch -s -d $(OUT)/engine -p1 < $(HERE)/m1-layer-batch.patch
	touch $@

$(OUT)/engine/m1_layer.o: $(OUT)/engine/.patched $(OUT)/.patched
	g++ -std=c++17 -O1 -c $(OUT)/engine/m1_layer.cpp -I$(TREE)/include -o $@

.PHONY: all
