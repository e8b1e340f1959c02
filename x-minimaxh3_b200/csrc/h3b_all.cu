// h3b_all.cu -- the whole library as one translation unit, so device globals
// (the status word) have a single definition without relocatable device code.
#include "quant.cu"
#include "gemm_i8.cu"
#include "w4a8.cu"
#include "attn_prep.cu"
#include "attn_mask.cu"
#include "attn.cu"
#include "ulysses.cu"
#include "adaln.cu"
#include "capi.cu"
