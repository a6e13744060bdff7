// wzyb200_all.cu -- the one CUDA translation unit of libwzyb200.so. The kernels share the device
// fault word (runtime.cu), so they are compiled together instead of with relocatable device code.
#include "runtime.cu"
#include "norm_rows.cu"
#include "head_rope.cu"
#include "gdn_norm.cu"
#include "swiglu.cu"
#include "gather.cu"
#include "hc_stream.cu"
#include "kv_append.cu"
#include "ple_block.cu"
#include "quant_act.cu"
#include "bundle.cu"
