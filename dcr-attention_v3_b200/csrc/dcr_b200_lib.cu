// dcr_b200_lib.cu — the single translation unit of libdcr_b200.so.
// The kernels share one device status word (g_device_status, dcr_common.cuh); building
// them as one unit keeps that a plain __device__ variable without relocatable device code.
#include "dcr_score.cu"
#include "dcr_select.cu"
#include "dcr_select_stream.cu"
#include "dcr_attend.cu"
#include "dcr_attend_union.cu"
#include "dcr_shard.cu"
#include "dcr_project.cu"
#include "dcr_rope.cu"
#include "dcr_decode_ops.cu"
#include "dcr_capi.cu"
#include "dcr_peer_capi.cu"
#include "dcr_noalloc.cu"
#include "dcr_runner.cu"
