// ovf_lib.cu — single translation unit of libovf_cuda.so.  The device-side
// error word (g_dev_error) is shared by every kernel, so the library is
// compiled as one unit instead of with relocatable device code.
#include "ovf_api.cu"
#include "ovf_quant.cu"
#include "ovf_gemv.cu"
#include "ovf_batched.cu"
#include "ovf_tc.cu"
#include "ovf_tc8.cu"
#include "ovf_tc6.cu"
#include "ovf_ops.cu"
#include "ovf_moe.cu"
#include "ovf_tp.cu"
#include "ovf_attn_cluster.cu"
#include "ovf_attn_group.cu"
#include "ovf_attn_exact.cu"
#include "ovf_attn_rows.cu"
#include "ovf_model.cu"
#include "ovf_noalloc.cu"
