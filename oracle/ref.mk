# Builds the reference's own kernels (read from the reference checkout, not copied)
# into oracle/_ref/libref_kernels.so for sm_100a. Only run where the checkout exists.
NVCC ?= nvcc
HERE := $(dir $(abspath $(lastword $(MAKEFILE_LIST))))
REF_CU ?= /root/reference/crates/paged-kv-cuda/kernels/kernels.cu

all: $(HERE)_ref/libref_kernels.so

$(HERE)_ref/libref_kernels.so: $(HERE)ref_launch.cu $(REF_CU)
	@mkdir -p $(HERE)_ref
	$(NVCC) -O3 -std=c++17 -gencode arch=compute_100a,code=sm_100a -lineinfo -Xcompiler -fPIC \
	    -Wno-deprecated-gpu-targets -shared -DREF_KERNELS_CU='"$(REF_CU)"' -o $@ $< -cudart static

.PHONY: all
