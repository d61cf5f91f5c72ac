# Compiles the reference's own GPU launcher from its sources, where they lie,
# with oracle/ref_shim.cu into oracle/_ref/libref_gpu.so (sm_100a).  Only the
# launcher and its kernel header are needed (src/gpu/gpu_kernel_launcher.cu,
# src/gpu/kernels/distance_kernels.cuh; CUDA runtime + cuBLAS); the rest of the
# reference needs Eigen, Boost, oneTBB and ibverbs and is not built.
# REF: the reference project's root (DVS_REFERENCE_ROOT, else where the build environment mounts it)
REF ?= $(or $(DVS_REFERENCE_ROOT),/root/reference)
HERE := $(dir $(abspath $(lastword $(MAKEFILE_LIST))))
NVCC ?= /usr/local/cuda/bin/nvcc
OUT := $(HERE)_ref/libref_gpu.so
FLAGS := -gencode arch=compute_100a,code=sm_100a -O3 -std=c++17 --expt-relaxed-constexpr --expt-extended-lambda \
         -Xcompiler -fPIC -I$(REF)/src

all: $(OUT)

$(OUT): $(HERE)ref_shim.cu $(REF)/src/gpu/gpu_kernel_launcher.cu $(REF)/src/gpu/kernels/distance_kernels.cuh
	mkdir -p $(HERE)_ref
	$(NVCC) $(FLAGS) -shared -o $@ $(HERE)ref_shim.cu $(REF)/src/gpu/gpu_kernel_launcher.cu -lcublas

.PHONY: all
