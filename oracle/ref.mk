# Builds the reference's own kernels (read from the reference checkout, not copied)
# into oracle/_ref/libref_kernels.so for sm_100a. PKV_REFERENCE_DIR names the
# checkout; where it is absent the recipe builds nothing (the prebuilt library,
# if any, is used as it is).
NVCC ?= nvcc
HERE := $(dir $(abspath $(lastword $(MAKEFILE_LIST))))
PKV_REFERENCE_DIR ?= /root/reference
REF_CU := $(PKV_REFERENCE_DIR)/crates/paged-kv-cuda/kernels/kernels.cu

ifeq ($(wildcard $(REF_CU)),)
all:
	@echo "oracle/ref.mk: no reference checkout at $(PKV_REFERENCE_DIR); skipping"
else
all: $(HERE)_ref/libref_kernels.so
endif

$(HERE)_ref/libref_kernels.so: $(HERE)ref_launch.cu $(REF_CU)
	@mkdir -p $(HERE)_ref
	$(NVCC) -O3 -std=c++17 -gencode arch=compute_100a,code=sm_100a -lineinfo -Xcompiler -fPIC \
	    -Wno-deprecated-gpu-targets -shared -DREF_KERNELS_CU='"$(REF_CU)"' -o $@ $< -cudart static

.PHONY: all
