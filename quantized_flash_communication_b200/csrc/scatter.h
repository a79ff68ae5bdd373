// Arguments of the GEMM epilogue that quantizes its output tile and stores it straight
// into the owning rank's reduce-scatter slot (the first phase of the two-shot quantized
// all-reduce, fused into the row-parallel o_proj / down_proj GEMMs).  Plain C++ so that
// host-only code can fill it.
#pragma once

#include <stdint.h>

#include "workspace.h"

namespace qfc {

struct ScatterArgs {
  char* base[kMaxRanks];  // every rank's workspace base (peer-mapped)
  int64_t rs_off;         // reduce-scatter region offset
  int64_t slot1;          // bytes per source slot
  int64_t pay1;           // payload bytes before the metadata in a slot
  int64_t chunk;          // elements per owner chunk of the flattened [M, N] output
  int rank, world;
  int gs_shift;           // log2(group size); the fused epilogue takes group size 128
  int sym, meta_fp32;
  uint32_t* epoch;        // this rank's fused-GEMM epoch counter (device)
  uint32_t* done_ctas;    // CTAs of the current launch that finished their stores (device)
};

}  // namespace qfc
