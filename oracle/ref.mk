# ref.mk -- builds the reference's own CPU implementation of the path (TEST INFRASTRUCTURE ONLY).
#
# Compiles the vendored ggml core + ggml-cpu backend of jmars/aubier (llama.cpp @ 50e3e3e4, under
# vendor/llama.cpp/ggml/ of the reference tree) directly from the reference's source files with
# gcc/g++, together with our own harness (ref_harness.c) that builds the unfused MLA decode graph
# of engine/m1_layer.cpp:443-502.  The reference's own CMake build is NOT used: this file lists the
# sources and the definitions that CMake would pass (GGML_USE_LLAMAFILE, GGML_USE_OPENMP) itself.
# The only configured file, ggml-version.h (two string macros), is written into the output folder.
#
# Nothing is copied out of the reference tree; every output goes to $(OUT) (oracle/_ref/),
# which is git-ignored.  Two ISA variants are built so the GPU box's host can pick the widest one
# it supports at run time: v3 (AVX2+FMA+F16C) and v4 (AVX-512 F/BW/CD/DQ/VL).
#
# usage: make -f oracle/ref.mk REF=<reference root> OUT=oracle/_ref -j8

REF ?= /nonexistent
OUT ?= oracle/_ref
GG  := $(REF)/vendor/llama.cpp/ggml

BASE_C   := ggml.c ggml-alloc.c ggml-quants.c
BASE_CXX := ggml.cpp ggml-backend.cpp ggml-backend-meta.cpp ggml-opt.cpp ggml-threading.cpp gguf.cpp
CPU_C    := ggml-cpu/ggml-cpu.c ggml-cpu/quants.c ggml-cpu/arch/x86/quants.c
CPU_CXX  := ggml-cpu/ggml-cpu.cpp ggml-cpu/repack.cpp ggml-cpu/hbm.cpp ggml-cpu/traits.cpp \
            ggml-cpu/amx/amx.cpp ggml-cpu/amx/mmq.cpp ggml-cpu/binary-ops.cpp \
            ggml-cpu/unary-ops.cpp ggml-cpu/vec.cpp ggml-cpu/ops.cpp \
            ggml-cpu/tiled/tiled.cpp ggml-cpu/tiled/tiled-kernel.cpp \
            ggml-cpu/llamafile/sgemm.cpp ggml-cpu/arch/x86/repack.cpp

DEFS := -DNDEBUG -D_GNU_SOURCE -D_XOPEN_SOURCE=600 -DGGML_USE_LLAMAFILE -DGGML_USE_OPENMP \
        -DGGML_USE_CPU -DGGML_SCHED_MAX_COPIES=4
INCS := -I$(OUT)/gen -I$(GG)/include -I$(GG)/src -I$(GG)/src/ggml-cpu
COMMON := -O3 -fPIC -fopenmp -pthread $(DEFS) $(INCS) -Wno-unused-result

ISA_v3 := -march=x86-64-v3
ISA_v4 := -march=x86-64-v4

VARIANTS := v3 v4

all: $(foreach v,$(VARIANTS),$(OUT)/libggml_ref_$(v).so)

$(OUT)/gen/ggml-version.h:
	@mkdir -p $(dir $@)
	@printf '#pragma once\n#define GGML_VERSION "0.26.0"\n#define GGML_COMMIT "50e3e3e4"\n' > $@

define variant
$(OUT)/obj_$(1)/%.c.o: $(GG)/src/%.c $(OUT)/gen/ggml-version.h
	@mkdir -p $$(dir $$@)
	gcc -std=gnu11 $(COMMON) $(ISA_$(1)) -c $$< -o $$@

$(OUT)/obj_$(1)/%.cpp.o: $(GG)/src/%.cpp $(OUT)/gen/ggml-version.h
	@mkdir -p $$(dir $$@)
	g++ -std=gnu++17 $(COMMON) $(ISA_$(1)) -c $$< -o $$@

$(OUT)/obj_$(1)/ref_harness.o: oracle/ref_harness.c $(OUT)/gen/ggml-version.h
	@mkdir -p $$(dir $$@)
	gcc -std=gnu11 $(COMMON) $(ISA_$(1)) -c $$< -o $$@

OBJS_$(1) := $(addprefix $(OUT)/obj_$(1)/,$(addsuffix .o,$(BASE_C) $(BASE_CXX) $(CPU_C) $(CPU_CXX))) \
             $(OUT)/obj_$(1)/ref_harness.o

$(OUT)/libggml_ref_$(1).so: $$(OBJS_$(1))
	g++ -shared -fopenmp -pthread -Wl,--no-undefined -o $$@ $$^ -lm
endef

$(foreach v,$(VARIANTS),$(eval $(call variant,$(v))))

.PHONY: all
