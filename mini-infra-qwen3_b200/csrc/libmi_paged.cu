// Unity translation unit of libmi_paged.so: one TU so that the device status word and the kernels
// share one module without relocatable device code.
#include "kv_scatter.cu"
#include "paged_decode.cu"
#include "paged_prefill_tc.cu"
#include "paged_prefill.cu"
#include "layer_ops.cu"
#include "api.cu"
#include "api_layers.cu"
#include "decode_meta.cu"
#include "peer.cu"
#include "api_static.cu"
