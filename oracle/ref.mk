# Builds oracle/_ref/libfrref.so: the reference's own Thor W4A4 path
# (src/fr_quant_act.cu, src/fr_repack.cu, src/fr_gemm_f32out.cu and
# include/fr_kernels.h, compiled unmodified where they lie) for sm_100a against
# the CUTLASS 4.5 headers shipped in the image, plus oracle/ref_shim.cu (C
# linkage).  Test infrastructure: used by tests/ (byte-for-byte pins of the
# W4A4 quantizer, the weight repack and its scale-factor atom layout, and the
# GEMM) and by bench.py's comparison leg, never by the product.
#   make -f oracle/ref.mk REF=/path/to/reference
REF     ?= /root/reference
PY_SP   ?= $(shell python3 -c 'import sysconfig; print(sysconfig.get_paths()["purelib"])')
CUTLASS ?= $(PY_SP)/flashinfer/data/cutlass
NVCC    ?= /usr/local/cuda/bin/nvcc
HERE    := $(dir $(lastword $(MAKEFILE_LIST)))
OUTDIR  := $(HERE)_ref
FLAGS   := -O3 -std=c++17 -gencode arch=compute_100a,code=sm_100a -Xcompiler -fPIC --expt-relaxed-constexpr \
           -DNDEBUG -I$(REF)/include -I$(CUTLASS)/include -I$(CUTLASS)/tools/util/include
SRCS    := $(REF)/src/fr_quant_act.cu $(REF)/src/fr_repack.cu $(REF)/src/fr_gemm_f32out.cu
OBJS    := $(OUTDIR)/fr_quant_act.o $(OUTDIR)/fr_repack.o $(OUTDIR)/fr_gemm_f32out.o $(OUTDIR)/ref_shim.o

all: $(OUTDIR)/libfrref.so

$(OUTDIR)/%.o: $(REF)/src/%.cu
	@mkdir -p $(OUTDIR)
	$(NVCC) $(FLAGS) -c -o $@ $<

$(OUTDIR)/ref_shim.o: $(HERE)ref_shim.cu
	@mkdir -p $(OUTDIR)
	$(NVCC) $(FLAGS) -c -o $@ $<

$(OUTDIR)/libfrref.so: $(OBJS)
	$(NVCC) -gencode arch=compute_100a,code=sm_100a -shared -o $@ $(OBJS) -lcudart

.PHONY: all
