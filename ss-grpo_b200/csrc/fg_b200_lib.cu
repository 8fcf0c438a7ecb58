// fg_b200_lib.cu -- single translation unit of libfgb200.so.
//
// The kernels share one device-side error word, so they are compiled as one
// unit (no relocatable device code is needed).
#include "fg_abi.cu"
#include "fg_sampling.cu"
#include "fg_tree.cu"
#include "fg_accept.cu"
#include "fg_layers.cu"
#include "fg_attention_tc.cu"
#include "fg_attention_tc2.cu"
#include "fg_attention.cu"
#include "fg_attention_noalloc.cu"
#include "fg_lmhead_tc.cu"
#include "fg_propose.cu"
#include "fg_chain.cu"
#include "fg_gemm_tc.cu"
