# fattn.mk -- builds upstream ggml-cuda for sm_100a as a comparator for the fused path: the
# reference's vendored llama.cpp FLASH_ATTN_EXT (ggml-cuda/fattn.cu:357-410, the mma.sync kernels of
# fattn-mma-f16.cuh) at the MLA shape DKQ = 576 / DV = 512, timed on the same B200 by
# fattn_compare.cpp.  It is measured, not built upon.
#
# Uses the patched tree of ggml.mk ($(TREE), run that first): every ggml-cuda/*.cu except the
# reference's HIP-flavoured M4 launchers (replaced there by m4-b200.cu), the tile / mma / mmq / mmf
# template instances and the f16-f16 vector FA instances (CMake's default set without the
# quantized caches this comparison does not use), then links one shared library with the patched
# ggml core + ggml-cpu objects of ggml.mk and the harness.  Objects go to $(OUT), the library and
# the harness to $(CMP) (both git-ignored; $(CMP) is 180 MB of sm_100a code, sent to the GPU box
# only for a comparator run).
#
# usage: make -f aubier_b200/ggml/fattn.mk OUT=aubier_b200/ggml/_build CMP=aubier_b200/ggml/_cmp -j8

OUT  ?= aubier_b200/ggml/_build
CMP  ?= aubier_b200/ggml/_cmp
HERE := aubier_b200/ggml
TREE := $(OUT)/ggml
CU   := $(TREE)/src/ggml-cuda
NVCC ?= nvcc

FA_DEFS := -DGGML_CUDA_FA_QUANTS=\"f16-f16\" \
           $(foreach k,Q4_0 Q4_1 Q5_0 Q5_1 Q8_0 BF16 F16,$(foreach v,Q4_0 Q4_1 Q5_0 Q5_1 Q8_0 BF16 F16,\
             -DGGML_CUDA_FA_$(k)_$(v)=$(if $(and $(filter F16,$(k)),$(filter F16,$(v))),1,0)))
CUDA_FLAGS := -std=c++17 -gencode arch=compute_100a,code=sm_100a -O3 -Xcompiler -fPIC \
              -DGGML_USE_CUDA -DGGML_CUDA_USE_GRAPHS -DGGML_SCHED_MAX_COPIES=4 $(FA_DEFS) \
              -I$(OUT)/gen -I$(TREE)/include -I$(TREE)/src -I$(CU) -Iinclude \
              -use_fast_math -extended-lambda

CU_SRCS := $(filter-out $(CU)/m4-wkb.cu $(CU)/m4-kqkv.cu $(CU)/m4-phase.cu,$(wildcard $(CU)/*.cu)) \
           $(wildcard $(CU)/template-instances/fattn-tile*.cu) \
           $(wildcard $(CU)/template-instances/fattn-mma*.cu) \
           $(wildcard $(CU)/template-instances/mmq*.cu) \
           $(wildcard $(CU)/template-instances/mmf*.cu) \
           $(CU)/template-instances/fattn-vec-instance-f16-f16.cu
CU_OBJS := $(patsubst $(CU)/%.cu,$(OUT)/cmp_obj/%.o,$(CU_SRCS))
GGML_OBJS := $(wildcard $(OUT)/obj/*.o $(OUT)/obj/*/*.o $(OUT)/obj/*/*/*.o $(OUT)/obj/*/*/*/*.o)
GGML_OBJS := $(filter-out $(OUT)/obj/m4b_ggml_check.o,$(GGML_OBJS))

all: $(CMP)/fattn_compare

$(OUT)/cmp_obj/%.o: $(CU)/%.cu
	@mkdir -p $(dir $@)
	$(NVCC) $(CUDA_FLAGS) -c $< -o $@

$(OUT)/cmp_obj/fattn_compare.o: $(HERE)/fattn_compare.cpp
	@mkdir -p $(dir $@)
	g++ -std=c++17 -O2 -I$(TREE)/include -I/usr/local/cuda/include -c $< -o $@

$(CMP)/libggml_cmp.so: $(CU_OBJS) $(GGML_OBJS) aubier_b200/libm4b.so
	$(NVCC) -shared -o $@ $(CU_OBJS) $(GGML_OBJS) -Laubier_b200 -lm4b -lcublas -lcublasLt \
	    -L/usr/local/cuda/lib64/stubs -lcuda \
	    -Xlinker -rpath -Xlinker '$$ORIGIN/../..'

$(CMP)/fattn_compare: $(OUT)/cmp_obj/fattn_compare.o $(CMP)/libggml_cmp.so
	g++ -o $@ $< -L$(CMP) -lggml_cmp -Wl,-rpath,'$$ORIGIN' -Wl,-rpath,'$$ORIGIN/../..' \
	    -L/usr/local/cuda/lib64 -lcudart -L/usr/local/cuda/lib64/stubs -lcuda -lpthread

.PHONY: all
