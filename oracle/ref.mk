# Builds the reference pdefa CPU engine (PDEFA1.0 + imageloader + pdefa C API)
# straight from its source files into oracle/_ref/libpdefa_ref.so.
#
# TEST INFRASTRUCTURE ONLY: the library built here is the parity checker and the
# timed CPU baseline. Nothing in the product links or loads it.
#
# Recipe notes
#  * No reference build system is run: this file lists the same sources as the
#    reference's PDEFA1.0/src/CMakeLists.txt:5-52 (+ AVX2 objects 114-122) and
#    imageloader/CMakeLists.txt:13-26, and compiles them with g++.
#  * The reference expects a CMake-configured header engine/version.hpp
#    (PDEFA1.0/cmake/version.hpp.in); this recipe writes the four version defines
#    itself into _ref/include/engine/version.hpp.
#  * AVX-512 is left out on purpose (PDEFA1.0/src/kernels/kernel_registry.cpp:33-43
#    would otherwise pick the 4x16 AVX-512 prototype over the AVX2 sgemm).
#  * Flags follow PDEFA1.0/cmake/CompilerFlags.cmake:34 and 43-49 (-O3,
#    -ffp-contract=fast, -fno-math-errno, -fno-trapping-math) with -mavx2 -mfma.
#
# Usage: make -f oracle/ref.mk REF=/path/to/reference [-j8]   (REF is required)

ifeq ($(strip $(REF)),)
$(error REF=<path of the pdefa reference checkout> is required)
endif
OUT      := $(dir $(lastword $(MAKEFILE_LIST)))_ref
OBJ      := $(OUT)/obj
LIB      := $(OUT)/libpdefa_ref.so
CXX      ?= g++

ENGINE   := $(REF)/PDEFA1.0
IMGL     := $(REF)/imageloader
NATIVE   := $(REF)/pdefa

ENGINE_SRCS := \
  core/tensor.cpp core/model.cpp core/session.cpp \
  memory/aligned_allocator.cpp memory/arena.cpp memory/memory_plan.cpp \
  runtime/cpu_info.cpp runtime/thread_pool.cpp runtime/affinity.cpp runtime/scheduler.cpp \
  runtime/random.cpp \
  kernels/kernel_registry.cpp kernels/generic/matmul_ref.cpp \
  ops/matmul.cpp ops/activation.cpp ops/conv2d.cpp ops/pooling.cpp ops/norm.cpp \
  ops/elementwise.cpp ops/concat.cpp ops/upsample.cpp ops/softmax.cpp ops/topk.cpp \
  ops/gather_elements.cpp \
  optimizer/graph_optimizer.cpp optimizer/layout_transform.cpp optimizer/quantization.cpp \
  loader/custom_loader.cpp api/engine_api.cpp \
  kernels/simd/avx2/matmul_avx2.cpp kernels/simd/avx2/activation_avx2.cpp \
  kernels/simd/avx2/conv2d_avx2.cpp kernels/simd/avx2/conv2d_winograd.cpp \
  kernels/simd/avx2/conv2d_gemm.cpp kernels/simd/avx2/conv2d_pointwise_avx2.cpp \
  kernels/simd/avx2/conv2d_direct_small_avx2.cpp

IMGL_SRCS := \
  src/loader.cpp src/preprocess.cpp \
  src/png/png_decoder.cpp src/png/png_chunks.cpp src/png/png_inflate.cpp \
  src/png/png_filters.cpp src/png/png_unpack.cpp \
  src/jpeg/jpeg_decoder.cpp src/jpeg/jpeg_markers.cpp src/jpeg/jpeg_huffman.cpp \
  src/jpeg/jpeg_idct.cpp src/jpeg/jpeg_color.cpp src/engine_api.cpp

CXXFLAGS := -std=c++20 -O3 -fPIC -mavx2 -mfma -ffp-contract=fast -fno-math-errno \
            -fno-trapping-math -funroll-loops -DNDEBUG -w \
            -DENGINE_PROFILING=1 -DENGINE_USE_AVX2=1 -DENGINE_USE_FMA=1 \
            -DENGINE_BUILDING_SHARED -DENGINE_SHARED -DPDEFA_BUILD \
            -I$(OUT)/include -I$(ENGINE)/include -I$(ENGINE)/src \
            -I$(IMGL)/include -I$(IMGL)/src/png -I$(IMGL)/src/jpeg -I$(NATIVE)/include

ENGINE_OBJS := $(patsubst %.cpp,$(OBJ)/engine/%.o,$(ENGINE_SRCS))
IMGL_OBJS   := $(patsubst %.cpp,$(OBJ)/imgl/%.o,$(IMGL_SRCS))
NATIVE_OBJS := $(OBJ)/native/pdefa_c_api.o
VERSION_HDR := $(OUT)/include/engine/version.hpp

all: $(LIB)

$(VERSION_HDR):
	@mkdir -p $(dir $@)
	@printf '#pragma once\n#define ENGINE_VERSION_MAJOR 1\n#define ENGINE_VERSION_MINOR 0\n#define ENGINE_VERSION_PATCH 0\n#define ENGINE_VERSION_STRING "1.0.0"\n#define ENGINE_USE_AVX2\n#define ENGINE_USE_FMA\n' > $@

$(OBJ)/engine/%.o: $(ENGINE)/src/%.cpp $(VERSION_HDR)
	@mkdir -p $(dir $@)
	$(CXX) $(CXXFLAGS) -c $< -o $@

$(OBJ)/imgl/%.o: $(IMGL)/%.cpp $(VERSION_HDR)
	@mkdir -p $(dir $@)
	$(CXX) $(CXXFLAGS) -c $< -o $@

$(OBJ)/native/pdefa_c_api.o: $(NATIVE)/src/pdefa_c_api.cpp $(VERSION_HDR)
	@mkdir -p $(dir $@)
	$(CXX) $(CXXFLAGS) -c $< -o $@

$(LIB): $(ENGINE_OBJS) $(IMGL_OBJS) $(NATIVE_OBJS)
	$(CXX) -shared -o $@ $^ -lpthread

clean:
	rm -rf $(OUT)

.PHONY: all clean
