// Single translation unit for all device code of libbeam_b200.so: the
// kernels share one device status word, so they are compiled together
// instead of with relocatable device code.
#include "page_ops.cu"
#include "attention.cu"
#include "attention_tma.cu"
#include "attention_umma.cu"
#include "attention_wide.cu"
#include "attention_narrow.cu"
#include "attention_tiles.cu"
#include "attn_api.cu"
#include "attn_noalloc.cu"
#include "model_ops.cu"
#include "select_ops.cu"
#include "gemm.cu"
#include "gemm_lt.cu"
#include "comm.cu"
