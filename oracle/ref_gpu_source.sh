#!/bin/sh
# Assembles the reference's CUDA kernel text as silvic-gpu's `kernel_source` does for NVRTC (crates/silvic-gpu/src/
# params.rs:30-53): its CUDA prelude, the shared capacities as #defines, common.h, kernels.kern. The reference's
# files are read where they lie; the result goes to oracle/_ref/ only (not committed).
set -e
if [ -z "$1" ]; then
  echo "usage: ref_gpu_source.sh <reference checkout> [output]" >&2
  exit 2
fi
REF=$1
OUT=${2:-_ref/ref_kernels.cuh}
K="$REF/crates/silvic-gpu/kernels"
{
  cat "$K/prelude_cuda.h"
  echo
  for d in "HIST_QUANT_BINS 8192" "HIST_FLOAT_BINS 4096" "REDUCE_THREADS 256" "SCAN_THREADS 256" \
           "LAMBDARANK_CAP_SMALL 64" "LAMBDARANK_CAP_MEDIUM 256" "LAMBDARANK_CAP_LARGE 1024" \
           "LAMBDARANK_THREADS_MAX 256" "HIST_SIDE_LEFT 1" "HIST_SIDE_RIGHT 2"; do
    set -- $d
    echo "#define $1 $2u"
  done
  cat "$K/common.h"
  echo
  cat "$K/kernels.kern"
} > "$OUT"
