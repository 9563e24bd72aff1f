// C-ABI entry points (include/prismyra_moe.h): argument checks, workspace carving, tensor-map encoding and the
// launch sequence of the routed-expert layer.  Nothing here allocates device memory or synchronises, except
// pm_moe_read_status.
#include <cudaTypedefs.h>
#include <limits.h>
#include <stdint.h>
#include <string.h>

#include <mutex>

#include "prismyra_moe.h"
#include "moe_internal.h"

namespace pm {

// ------------------------------------------------------------------------------------------- tensor maps
static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
static std::once_flag g_encode_once;

bool encode_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elem_bytes, uint64_t inner,
                    uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer) {
    std::call_once(g_encode_once, [] {
        cudaDriverEntryPointQueryResult q;
        void* fn = nullptr;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    });
    if (g_encode == nullptr) return false;
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    (void)elem_bytes;
    CUresult r = g_encode(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// ------------------------------------------------------------------------------------------- device facts
struct DeviceInfo {
    int sms = 0;
    int ok = -1;  // -1 unknown, 0 not sm_100, 1 sm_100
};
static DeviceInfo g_dev[64];
static std::mutex g_dev_mu;

static int current_device_info(DeviceInfo* out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return PM_ERR_CUDA;
    std::lock_guard<std::mutex> lk(g_dev_mu);
    DeviceInfo& d = g_dev[dev];
    if (d.ok < 0) {
        int major = 0, minor = 0, sms = 0;
        if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
            return PM_ERR_CUDA;
        d.ok = (major == 10 && minor == 0) ? 1 : 0;
        d.sms = sms;
    }
    *out = d;
    return d.ok ? PM_OK : PM_ERR_DEVICE;
}

// ------------------------------------------------------------------------------------------- workspace
constexpr int kRegions = PM_WS_SCHED + 1;

struct Layout {
    size_t off[kRegions];
    size_t len[kRegions];
    size_t total;
    int max_slots;
};

static size_t align256(size_t v) { return (v + 255) & ~(size_t)255; }

static int max_slots_of(int T, int E, int k) {
    const long s = (long)T * k + (long)E * (kBlockM - 1);
    return (int)((s + kBlockM - 1) / kBlockM * kBlockM);
}

static Layout layout_of(int T, int H, int I, int E, int k, int fmt) {
    Layout L;
    const long n = (long)T * k;
    const int ms = max_slots_of(T, E, k);
    const int chunks = n > 0 ? align_chunks(n) : 1;
    const bool fp4 = fmt == PM_FMT_NVFP4;
    L.len[PM_WS_STATUS] = 4 * sizeof(int32_t);
    L.len[PM_WS_LOGITS] = (size_t)T * E * 2;
    L.len[PM_WS_TOPK_W] = (size_t)n * 4;
    L.len[PM_WS_TOPK_IDS] = (size_t)n * 4;
    L.len[PM_WS_COUNTS] = (size_t)chunks * E * 4;
    L.len[PM_WS_EXPERT_OFF] = (size_t)(E + 1) * 4;
    L.len[PM_WS_SORTED] = (size_t)ms * 4;
    L.len[PM_WS_EXPERT_IDS] = (size_t)(ms / kBlockM) * 4;
    L.len[PM_WS_NUM_POST_PAD] = 4;
    L.len[PM_WS_A1] = (size_t)ms * (fp4 ? H / 2 : H);
    L.len[PM_WS_A1_SCALE] = (size_t)ms * (fp4 ? H / 16 : (H / 128) * 4);
    L.len[PM_WS_A2] = (size_t)ms * (fp4 ? I / 2 : I);
    L.len[PM_WS_A2_SCALE] = (size_t)ms * (fp4 ? I / 16 : (I / 128) * 4);
    L.len[PM_WS_C3] = (size_t)n * H * 2;
    L.len[PM_WS_SLOT_OF] = (size_t)n * 4;
    L.len[PM_WS_ROUTER_PART] = router_split_bytes(T, H, E);
    L.len[PM_WS_SCHED] = (size_t)small_sched_ints(ms / kBlockM) * 4;
    size_t o = 0;
    for (int r = 0; r < kRegions; ++r) {
        L.off[r] = o;
        o = align256(o + L.len[r]);
    }
    L.total = o;
    L.max_slots = ms;
    return L;
}

static bool a16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

static int check_dims(int T, int H, int I, int E, int k) {
    if (T < 0 || H <= 0 || I <= 0 || E <= 0 || k <= 0) return PM_ERR_INVALID;
    if (H % 256 != 0 || I % 128 != 0 || k > kMaxTopK || k > E || E > kMaxExperts) return PM_ERR_SHAPE;
    if ((long)T * k > (1L << 30)) return PM_ERR_SHAPE;
    return PM_OK;
}

static int cuda_status(cudaError_t e) { return e == cudaSuccess ? PM_OK : PM_ERR_CUDA; }

// The activation-scale rule (e4m3_group_scale) a flags word selects, or -1 for an invalid word.
static int scale_rule_of(int flags) {
    switch (flags) {
        case 0: return kScaleDiv;
        case PM_FLAG_ACT_SCALE_UE8M0: return kScaleUe8m0;
        case PM_FLAG_ACT_SCALE_RCP: return kScaleRcp;
        default: return -1;
    }
}

static GemmArgs gemm_args_common(const float* a_s, const float* b_s, const int32_t* expert_ids,
                                 const int32_t* npp, int n_total, int K, int n_tiles, int max_slots, int inter,
                                 int32_t* err) {
    GemmArgs g;
    memset(&g, 0, sizeof(g));
    g.a_scale = a_s;
    g.b_scale = b_s;
    g.expert_ids = expert_ids;
    g.num_post_pad = npp;
    g.n_total = n_total;
    g.K = K;
    g.n_tiles = n_tiles;
    g.max_tiles = (max_slots / kBlockM) * n_tiles;
    g.inter = inter;
    g.err = err;
    return g;
}

}  // namespace pm

using namespace pm;

extern "C" {

int pm_moe_abi_version(void) { return 1; }

const char* pm_moe_status_string(int status) {
    switch (status) {
        case PM_OK: return "ok";
        case PM_ERR_INVALID: return "invalid argument (NULL pointer or negative size)";
        case PM_ERR_SHAPE: return "unsupported shape (need H%256==0, I%128==0, 1<=k<=16, k<=E<=256)";
        case PM_ERR_ALIGN: return "pointer not 16-byte aligned";
        case PM_ERR_WORKSPACE: return "workspace too small";
        case PM_ERR_CUDA: return "CUDA launch or driver call failed";
        case PM_ERR_DEVICE: return "current device is not sm_100 (B200)";
        case PM_ERR_TIMEOUT: return "a kernel gave up on a bounded wait";
        case PM_ERR_TOO_LARGE: return "beyond the no-allocation entry point's fixed scratch (T*k <= 2^20, E <= 256)";
        default: return "unknown status";
    }
}

int pm_moe_max_slots(int T, int E, int k) { return max_slots_of(T, E, k); }

size_t pm_moe_workspace_bytes(int T, int H, int I, int E, int k, int fmt) {
    if (check_dims(T, H, I, E, k) != PM_OK) return 0;
    return layout_of(T, H, I, E, k, fmt).total;
}

int pm_moe_workspace_region(int T, int H, int I, int E, int k, int fmt, int region, size_t* offset, size_t* bytes) {
    const int st = check_dims(T, H, I, E, k);
    if (st != PM_OK) return st;
    if (region < 0 || region >= kRegions || offset == nullptr || bytes == nullptr) return PM_ERR_INVALID;
    const Layout L = layout_of(T, H, I, E, k, fmt);
    *offset = L.off[region];
    *bytes = L.len[region];
    return PM_OK;
}

int pm_moe_router_topk(const void* x, const void* router_w, const float* bias, int T, int H, int E, int k,
                       void* logits, float* topk_w, int32_t* topk_ids, pm_stream_t stream) {
    if (T < 0 || H <= 0 || E <= 0 || k <= 0) return PM_ERR_INVALID;
    if (H % 128 != 0 || E > kMaxExperts || k > kMaxTopK || k > E) return PM_ERR_SHAPE;
    if (T == 0) return PM_OK;
    if (!x || !router_w || !topk_w || !topk_ids || !logits) return PM_ERR_INVALID;
    if (!a16(x) || !a16(router_w) || !a16(logits)) return PM_ERR_ALIGN;
    DeviceInfo d;
    const int st = current_device_info(&d);
    if (st != PM_OK) return st;
    return cuda_status(
        launch_router_topk(x, router_w, bias, T, H, E, k, logits, topk_w, topk_ids, nullptr, (cudaStream_t)stream));
}

int pm_moe_topk(const void* logits, const float* bias, int T, int E, int k, float* topk_w, int32_t* topk_ids,
                pm_stream_t stream) {
    if (T < 0 || E <= 0 || k <= 0) return PM_ERR_INVALID;
    if (E > kMaxExperts || k > kMaxTopK || k > E) return PM_ERR_SHAPE;
    if (T == 0) return PM_OK;
    if (!logits || !topk_w || !topk_ids) return PM_ERR_INVALID;
    DeviceInfo d;
    const int st = current_device_info(&d);
    if (st != PM_OK) return st;
    return cuda_status(launch_topk(logits, bias, T, E, k, topk_w, topk_ids, (cudaStream_t)stream));
}

size_t pm_moe_align_workspace_bytes(int T, int k, int E) {
    if (T < 0 || k <= 0 || E <= 0 || E > 1024) return 0;
    const long n = (long)T * k;
    if (n > INT_MAX) return 0;  // the kernels index the flat pairs with 32-bit integers
    return (size_t)(n > 0 ? align_chunks(n) : 1) * E * 4;
}

int pm_moe_align(const int32_t* topk_ids, int T, int k, int E, int32_t* sorted_ids, int32_t* expert_ids,
                 int32_t* num_post_pad, int32_t* expert_off, int32_t* slot_of, void* workspace,
                 size_t workspace_bytes, pm_stream_t stream) {
    if (T < 0 || k <= 0 || E <= 0 || E > 1024) return PM_ERR_INVALID;
    if (!sorted_ids || !expert_ids || !num_post_pad || !workspace || (T > 0 && !topk_ids)) return PM_ERR_INVALID;
    const long n = (long)T * k;
    if (n > INT_MAX) return PM_ERR_SHAPE;
    if (workspace_bytes < pm_moe_align_workspace_bytes(T, k, E)) return PM_ERR_WORKSPACE;
    DeviceInfo d;
    const int st = current_device_info(&d);
    if (st != PM_OK) return st;
    return cuda_status(launch_align(topk_ids, (int)n, E, static_cast<int32_t*>(workspace), sorted_ids, expert_ids,
                                    num_post_pad, expert_off, slot_of, (cudaStream_t)stream));
}

int pm_moe_quant_fp8(const void* x, int T, int H, int k, const int32_t* slot_of, uint8_t* a_q, float* a_s,
                     pm_stream_t stream) {
    return pm_moe_quant_fp8_ex(x, T, H, k, slot_of, a_q, a_s, 0, stream);
}

int pm_moe_quant_fp8_ex(const void* x, int T, int H, int k, const int32_t* slot_of, uint8_t* a_q, float* a_s,
                        int flags, pm_stream_t stream) {
    if (T < 0 || H <= 0 || (slot_of != nullptr && k <= 0) || scale_rule_of(flags) < 0) return PM_ERR_INVALID;
    if (H % 128 != 0) return PM_ERR_SHAPE;
    if (T == 0) return PM_OK;
    if (!x || !a_q || !a_s) return PM_ERR_INVALID;
    if (!a16(x) || !a16(a_q)) return PM_ERR_ALIGN;
    DeviceInfo d;
    const int st = current_device_info(&d);
    if (st != PM_OK) return st;
    return cuda_status(launch_quant_fp8(x, T, H, k, slot_of, a_q, a_s, (cudaStream_t)stream, scale_rule_of(flags)));
}

// The few-tokens-per-expert GEMMs (weights as the 128-row MMA operand): used when T*k <= 32 E.
static bool use_small_gemm(long n_valid, int H, int I, int E) {
    return n_valid <= (long)kSmallTokensPerExpert * E && gemm_fp8_small_fits(0, H) && gemm_fp8_small_fits(1, I);
}

static int small_gemm_fp8(int mode, const uint8_t* a_q, const float* a_s, const uint8_t* w, const float* w_s,
                          const int32_t* expert_ids, const int32_t* npp, const int32_t* sorted_ids,
                          const float* topk_w, int max_slots, int n_valid, int H, int I, int E, uint8_t* out_q,
                          float* out_s, void* c3, int32_t* err, int sms, cudaStream_t s, int scale_rule = 0) {
    const int K = mode == 0 ? H : I, n_total = mode == 0 ? 2 * I : H;
    CUtensorMap tt, tw;
    if (!encode_tmap_2d_u8(&tt, a_q, (uint64_t)K, (uint64_t)max_slots, (uint64_t)K, 128, 32) ||
        !encode_tmap_2d_u8(&tw, w, (uint64_t)K, (uint64_t)E * n_total, (uint64_t)K, 128, 128))
        return PM_ERR_CUDA;
    SmallGemmArgs g;
    memset(&g, 0, sizeof(g));
    g.a_scale = a_s;
    g.b_scale = w_s;
    g.expert_ids = expert_ids;
    g.num_post_pad = npp;
    g.sorted_ids = sorted_ids;
    g.n_valid = n_valid;
    g.n_total = n_total;
    g.K = K;
    g.n_tiles = mode == 0 ? I / 128 : H / 256;  // down units are 256 hidden rows
    g.max_units = (max_slots / kBlockM) * g.n_tiles;
    g.inter = I;
    g.out_q = out_q;
    g.out_s = out_s;
    g.topk_w = topk_w;
    g.c3 = static_cast<__nv_bfloat16*>(c3);
    g.scale_rule = scale_rule;
    g.err = err;
    return cuda_status(launch_gemm_fp8_small(mode, tt, tw, g, sms, s));
}

// Both few-tokens-per-expert GEMMs in one launch (the forward's path when use_small_gemm holds); sched has been
// zeroed by the quantisation launch.
static int small_fused_fp8(const uint8_t* a1, const float* a1s, const uint8_t* w1, const float* w1_s, uint8_t* a2,
                           float* a2s, const uint8_t* w2, const float* w2_s, const int32_t* expert_ids,
                           const int32_t* npp, const int32_t* sorted_ids, const float* topk_w, int max_slots,
                           int n_valid, int H, int I, int E, void* c3, int32_t* sched, int32_t* err, int sms,
                           cudaStream_t s, int scale_rule) {
    CUtensorMap t1, tw1, t2, tw2;
    if (!encode_tmap_2d_u8(&t1, a1, (uint64_t)H, (uint64_t)max_slots, (uint64_t)H, 128, 32) ||
        !encode_tmap_2d_u8(&tw1, w1, (uint64_t)H, (uint64_t)E * 2 * I, (uint64_t)H, 128, 128) ||
        !encode_tmap_2d_u8(&t2, a2, (uint64_t)I, (uint64_t)max_slots, (uint64_t)I, 128, 32) ||
        !encode_tmap_2d_u8(&tw2, w2, (uint64_t)I, (uint64_t)E * H, (uint64_t)I, 128, 128))
        return PM_ERR_CUDA;
    SmallGemmArgs g[2];
    memset(g, 0, sizeof(g));
    for (int m = 0; m < 2; ++m) {
        g[m].expert_ids = expert_ids;
        g[m].num_post_pad = npp;
        g[m].sorted_ids = sorted_ids;
        g[m].n_valid = n_valid;
        g[m].inter = I;
        g[m].scale_rule = scale_rule;
        g[m].err = err;
    }
    g[0].a_scale = a1s;
    g[0].b_scale = w1_s;
    g[0].n_total = 2 * I;
    g[0].K = H;
    g[0].n_tiles = I / 128;
    g[0].out_q = a2;
    g[0].out_s = a2s;
    g[0].prefetch_units = E * (I / 128);
    g[1].a_scale = a2s;
    g[1].b_scale = w2_s;
    g[1].n_total = H;
    g[1].K = I;
    g[1].n_tiles = H / 256;
    g[1].topk_w = topk_w;
    g[1].c3 = static_cast<__nv_bfloat16*>(c3);
    for (int m = 0; m < 2; ++m) g[m].max_units = (max_slots / kBlockM) * g[m].n_tiles;
    return cuda_status(launch_gemm_fp8_small_fused(t1, tw1, t2, tw2, g[0], g[1], sched, sms, s));
}

static int gemm1_fp8_run(const uint8_t* a_q, const float* a_s, const uint8_t* w1, const float* w1_s,
                         const int32_t* expert_ids, const int32_t* num_post_pad, int max_slots, int H, int I, int E,
                         uint8_t* out_q, float* out_s, int32_t* err, pm_stream_t stream, int scale_rule);

int pm_moe_gemm1_fp8(const uint8_t* a_q, const float* a_s, const uint8_t* w1, const float* w1_s,
                     const int32_t* expert_ids, const int32_t* num_post_pad, int max_slots, int H, int I, int E,
                     uint8_t* out_q, float* out_s, int32_t* err, pm_stream_t stream) {
    return gemm1_fp8_run(a_q, a_s, w1, w1_s, expert_ids, num_post_pad, max_slots, H, I, E, out_q, out_s, err, stream,
                         0);
}

static int gemm1_fp8_run(const uint8_t* a_q, const float* a_s, const uint8_t* w1, const float* w1_s,
                         const int32_t* expert_ids, const int32_t* num_post_pad, int max_slots, int H, int I, int E,
                         uint8_t* out_q, float* out_s, int32_t* err, pm_stream_t stream, int scale_rule) {
    int st = check_dims(0, H, I, E, 1);
    if (st != PM_OK) return st;
    if (max_slots < 0 || max_slots % kBlockM != 0) return PM_ERR_SHAPE;
    if (max_slots == 0) return PM_OK;
    if (!a_q || !a_s || !w1 || !w1_s || !expert_ids || !num_post_pad || !out_q || !out_s) return PM_ERR_INVALID;
    if (!a16(a_q) || !a16(w1) || !a16(out_q)) return PM_ERR_ALIGN;
    DeviceInfo d;
    st = current_device_info(&d);
    if (st != PM_OK) return st;
    CUtensorMap ta, tb;
    if (!encode_tmap_2d_u8(&ta, a_q, (uint64_t)H, (uint64_t)max_slots, (uint64_t)H, 128, 128) ||
        !encode_tmap_2d_u8(&tb, w1, (uint64_t)H, (uint64_t)E * 2 * I, (uint64_t)H, 128, 128))
        return PM_ERR_CUDA;
    GemmArgs g = gemm_args_common(a_s, w1_s, expert_ids, num_post_pad, 2 * I, H, I / 128, max_slots, I, err);
    g.out_q = out_q;
    g.out_s = out_s;
    g.scale_rule = scale_rule;
    return cuda_status(launch_gemm_fp8(0, ta, tb, g, d.sms, (cudaStream_t)stream));
}

int pm_moe_gemm2_fp8(const uint8_t* a_q, const float* a_s, const uint8_t* w2, const float* w2_s,
                     const int32_t* expert_ids, const int32_t* num_post_pad, const int32_t* sorted_ids,
                     const float* topk_w, int max_slots, int T, int k, int H, int I, int E, void* c3, int32_t* err,
                     pm_stream_t stream) {
    int st = check_dims(T, H, I, E, k);
    if (st != PM_OK) return st;
    if (max_slots < 0 || max_slots % kBlockM != 0) return PM_ERR_SHAPE;
    if (max_slots == 0 || T == 0) return PM_OK;
    if (!a_q || !a_s || !w2 || !w2_s || !expert_ids || !num_post_pad || !sorted_ids || !topk_w || !c3)
        return PM_ERR_INVALID;
    if (!a16(a_q) || !a16(w2) || !a16(c3)) return PM_ERR_ALIGN;
    DeviceInfo d;
    st = current_device_info(&d);
    if (st != PM_OK) return st;
    CUtensorMap ta, tb;
    if (!encode_tmap_2d_u8(&ta, a_q, (uint64_t)I, (uint64_t)max_slots, (uint64_t)I, 128, 128) ||
        !encode_tmap_2d_u8(&tb, w2, (uint64_t)I, (uint64_t)E * H, (uint64_t)I, 128, 128))
        return PM_ERR_CUDA;
    // (the small kernel copies the activation scales in bulk: 16-byte aligned rows of scales)
    if (use_small_gemm((long)T * k, H, I, E) && a16(a_s))
        return small_gemm_fp8(1, a_q, a_s, w2, w2_s, expert_ids, num_post_pad, sorted_ids, topk_w, max_slots, T * k,
                              H, I, E, nullptr, nullptr, c3, err, d.sms, (cudaStream_t)stream);
    GemmArgs g = gemm_args_common(a_s, w2_s, expert_ids, num_post_pad, H, I, H / 256, max_slots, I, err);
    g.sorted_ids = sorted_ids;
    g.topk_w = topk_w;
    g.c3 = static_cast<__nv_bfloat16*>(c3);
    g.n_valid = T * k;
    return cuda_status(launch_gemm_fp8(1, ta, tb, g, d.sms, (cudaStream_t)stream));
}

int pm_moe_scatter_rows(const void* src, int rows, int row_bytes, int src_stride, const int32_t* dst_index,
                        void* dst, int dst_stride, pm_stream_t stream) {
    if (rows < 0 || row_bytes <= 0 || src_stride < row_bytes || dst_stride < row_bytes) return PM_ERR_INVALID;
    if (row_bytes % 16 || src_stride % 16 || dst_stride % 16) return PM_ERR_ALIGN;
    if (rows == 0) return PM_OK;
    if (!src || !dst_index || !dst) return PM_ERR_INVALID;
    if (!a16(src) || !a16(dst)) return PM_ERR_ALIGN;
    DeviceInfo d;
    const int st = current_device_info(&d);
    if (st != PM_OK) return st;
    return cuda_status(
        launch_scatter_rows(src, rows, row_bytes, src_stride, dst_index, dst, dst_stride, (cudaStream_t)stream));
}

int pm_moe_combine(const void* c3, const int32_t* row_of, int T, int k, int H, void* out, pm_stream_t stream) {
    if (T < 0 || k <= 0 || H <= 0) return PM_ERR_INVALID;
    if (H % 8 != 0) return PM_ERR_SHAPE;
    if (T == 0) return PM_OK;
    if (!c3 || !out) return PM_ERR_INVALID;
    if (!a16(c3) || !a16(out)) return PM_ERR_ALIGN;
    DeviceInfo d;
    const int st = current_device_info(&d);
    if (st != PM_OK) return st;
    return cuda_status(launch_combine(c3, row_of, T, k, H, out, (cudaStream_t)stream));
}

// The routed layer; with add, the final sum adds add[t] (after waiting on add_ready when given).
static int forward_fp8_impl(const void* x, const void* router_w, const void* logits, const uint8_t* w1,
                            const float* w1_s, const uint8_t* w2, const float* w2_s, int T, int H, int I, int E,
                            int k, const void* add, cudaEvent_t add_ready, void* out, void* workspace,
                            size_t workspace_bytes, pm_stream_t stream, bool clear_status, int scale_rule = 0,
                            const float* bias = nullptr) {
    int st = check_dims(T, H, I, E, k);
    if (st != PM_OK) return st;
    if (T == 0) return PM_OK;
    if (!x || !w1 || !w1_s || !w2 || !w2_s || !out || !workspace || (!router_w && !logits)) return PM_ERR_INVALID;
    if (!a16(x) || !a16(w1) || !a16(w2) || !a16(out) || !a16(workspace) || (router_w && !logits && !a16(router_w)))
        return PM_ERR_ALIGN;
    const Layout L = layout_of(T, H, I, E, k, PM_FMT_FP8);
    if (workspace_bytes < L.total) return PM_ERR_WORKSPACE;
    DeviceInfo d;
    st = current_device_info(&d);
    if (st != PM_OK) return st;
    cudaStream_t s = (cudaStream_t)stream;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    auto R = [&](int r) { return ws + L.off[r]; };
    float* router_part = L.len[PM_WS_ROUTER_PART] > 0 ? reinterpret_cast<float*>(R(PM_WS_ROUTER_PART)) : nullptr;
    int32_t* status = reinterpret_cast<int32_t*>(R(PM_WS_STATUS));
    float* topk_w = reinterpret_cast<float*>(R(PM_WS_TOPK_W));
    int32_t* topk_ids = reinterpret_cast<int32_t*>(R(PM_WS_TOPK_IDS));
    int32_t* sorted = reinterpret_cast<int32_t*>(R(PM_WS_SORTED));
    int32_t* expert_ids = reinterpret_cast<int32_t*>(R(PM_WS_EXPERT_IDS));
    int32_t* npp = reinterpret_cast<int32_t*>(R(PM_WS_NUM_POST_PAD));
    uint8_t* a1 = R(PM_WS_A1);
    float* a1s = reinterpret_cast<float*>(R(PM_WS_A1_SCALE));
    uint8_t* a2 = R(PM_WS_A2);
    float* a2s = reinterpret_cast<float*>(R(PM_WS_A2_SCALE));
    void* c3 = R(PM_WS_C3);

    // The status words start at zero: with the router projection, its kernel (the forward's first) zeroes them, so
    // that the previous forward's last kernel and this forward's first still overlap; with given logits, a memset.
    int32_t* clear = clear_status && logits == nullptr ? status : nullptr;
    if (clear_status && clear == nullptr && cudaMemsetAsync(status, 0, L.len[PM_WS_STATUS], s) != cudaSuccess)
        return PM_ERR_CUDA;
    int32_t* slot_of = reinterpret_cast<int32_t*>(R(PM_WS_SLOT_OF));
    // Both few-token GEMMs in one launch once most experts are hit (T*k >= 2E); with fewer pairs nearly every down
    // unit would wait for its block's few gate_up units, and two launches are faster.
    const bool fused = use_small_gemm((long)T * k, H, I, E) && (long)T * k >= 2L * E &&
                       gemm_fp8_small_fused_fits(H, I) && a16(a1s) && a16(a2s);
    int32_t* sched = reinterpret_cast<int32_t*>(R(PM_WS_SCHED));
    int32_t* zero = fused ? sched : nullptr;
    const int zero_n = fused ? small_sched_ints(L.max_slots / kBlockM) : 0;
    cudaError_t e;
    if ((long)T * k >= kFrontMinIndices && (long)T * k <= kFrontMaxIndices) {
        // few tokens: the top-k, the alignment and the quantisation in one launch after the router projection
        const bool split = logits == nullptr && router_part != nullptr && router_split_bytes(T, H, E) > 0;
        if (logits == nullptr) {
            e = launch_router_topk(x, router_w, bias, T, H, E, k, R(PM_WS_LOGITS), topk_w, topk_ids, status, s,
                                   router_part, false, clear);
            if (e != cudaSuccess) return PM_ERR_CUDA;
        }
        const void* lg_in = split ? nullptr : (logits != nullptr ? logits : R(PM_WS_LOGITS));
        e = launch_front_small(split ? router_part : nullptr, router_chunks(H), lg_in, R(PM_WS_LOGITS), bias, T, E,
                               k, topk_w, topk_ids, sorted, expert_ids, npp,
                               reinterpret_cast<int32_t*>(R(PM_WS_EXPERT_OFF)), slot_of, x, H, a1, a1s, scale_rule,
                               zero, zero_n, status + 2, status, s);
        if (e != cudaSuccess) return PM_ERR_CUDA;
    } else {
        if (logits != nullptr)
            e = launch_topk(logits, bias, T, E, k, topk_w, topk_ids, s);
        else
            e = launch_router_topk(x, router_w, bias, T, H, E, k, R(PM_WS_LOGITS), topk_w, topk_ids, status, s,
                                   router_part, true, clear);
        if (e != cudaSuccess) return PM_ERR_CUDA;
        e = launch_align(topk_ids, T * k, E, reinterpret_cast<int32_t*>(R(PM_WS_COUNTS)), sorted, expert_ids, npp,
                         reinterpret_cast<int32_t*>(R(PM_WS_EXPERT_OFF)), slot_of, s);
        if (e != cudaSuccess) return PM_ERR_CUDA;
        e = launch_quant_fp8(x, T, H, k, slot_of, a1, a1s, s, scale_rule, zero, zero_n);
        if (e != cudaSuccess) return PM_ERR_CUDA;
    }
    if (fused) {
        st = small_fused_fp8(a1, a1s, w1, w1_s, a2, a2s, w2, w2_s, expert_ids, npp, sorted, topk_w, L.max_slots,
                             T * k, H, I, E, c3, sched, status, d.sms, s, scale_rule);
    } else {
        if (use_small_gemm((long)T * k, H, I, E))
            st = small_gemm_fp8(0, a1, a1s, w1, w1_s, expert_ids, npp, sorted, nullptr, L.max_slots, T * k, H, I, E,
                                a2, a2s, nullptr, status, d.sms, s, scale_rule);
        else
            st = gemm1_fp8_run(a1, a1s, w1, w1_s, expert_ids, npp, L.max_slots, H, I, E, a2, a2s, status, stream,
                               scale_rule);
        if (st != PM_OK) return st;
        st = pm_moe_gemm2_fp8(a2, a2s, w2, w2_s, expert_ids, npp, sorted, topk_w, L.max_slots, T, k, H, I, E, c3,
                              status, stream);
    }
    if (st != PM_OK) return st;
    if (add_ready != nullptr && cudaStreamWaitEvent(s, add_ready, 0) != cudaSuccess) return PM_ERR_CUDA;
    return cuda_status(launch_combine(c3, nullptr, T, k, H, out, s, add));
}

int pm_moe_forward_fp8(const void* x, const void* router_w, const void* logits, const uint8_t* w1,
                       const float* w1_s, const uint8_t* w2, const float* w2_s, int T, int H, int I, int E, int k,
                       void* out, void* workspace, size_t workspace_bytes, pm_stream_t stream) {
    return forward_fp8_impl(x, router_w, logits, w1, w1_s, w2, w2_s, T, H, I, E, k, nullptr, nullptr, out,
                            workspace, workspace_bytes, stream, true);
}

int pm_moe_forward_fp8_ex(const void* x, const void* router_w, const void* logits, const float* bias,
                          const uint8_t* w1, const float* w1_s, const uint8_t* w2, const float* w2_s, int T, int H,
                          int I, int E, int k, int flags, void* out, void* workspace, size_t workspace_bytes,
                          pm_stream_t stream) {
    const int rule = scale_rule_of(flags);
    if (rule < 0) return PM_ERR_INVALID;
    return forward_fp8_impl(x, router_w, logits, w1, w1_s, w2, w2_s, T, H, I, E, k, nullptr, nullptr, out,
                            workspace, workspace_bytes, stream, true, rule, bias);
}

// ------------------------------------------------------------------------------------------- shared expert
// Scratch of the shared expert: status word, gate [T], the one-expert plan, the quantised input rows, the
// quantised silu*mul rows, and (for the whole block) the shared output before it is added to the routed sum.
struct SharedLayout {
    size_t status, gate, expert_ids, npp, xq, xs, a2, a2s, out, total;
    int rows;  // T rounded up to the 128-row blocks
};

// One non-blocking side stream and a fork/join event pair per (thread, device), created on first use and kept
// for the life of the thread (make the first call before any stream capture begins).
struct SideStream {
    cudaStream_t stream = nullptr;
    cudaEvent_t fork = nullptr, join = nullptr;
};

static SideStream* side_stream() {
    thread_local SideStream per_device[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    SideStream& ss = per_device[dev];
    if (ss.stream == nullptr) {
        if (cudaStreamCreateWithFlags(&ss.stream, cudaStreamNonBlocking) != cudaSuccess) return nullptr;
        if (cudaEventCreateWithFlags(&ss.fork, cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&ss.join, cudaEventDisableTiming) != cudaSuccess)
            return nullptr;
    }
    return &ss;
}

static SharedLayout shared_layout_of(int T, int H, int Is, bool with_out) {
    SharedLayout L;
    const int rows = (T + kBlockM - 1) / kBlockM * kBlockM;
    size_t o = 0;
    auto take = [&](size_t bytes) { const size_t at = o; o = align256(o + bytes); return at; };
    L.status = take(4 * sizeof(int32_t));
    L.gate = take((size_t)T * 4);
    L.expert_ids = take((size_t)(rows / kBlockM) * 4);
    L.npp = take(4);
    L.xq = take((size_t)rows * H);
    L.xs = take((size_t)rows * (H / 128) * 4);
    L.a2 = take((size_t)rows * Is);
    L.a2s = take((size_t)rows * (Is / 128) * 4);
    L.out = with_out ? take((size_t)T * H * 2) : 0;
    L.total = o;
    L.rows = rows;
    return L;
}

static int check_shared_dims(int T, int H, int Is) {
    if (T < 0 || H <= 0 || Is <= 0) return PM_ERR_INVALID;
    if (H % 256 != 0 || Is % 128 != 0 || (long)T * H > (1L << 34)) return PM_ERR_SHAPE;
    return PM_OK;
}

// sigmoid(gate(x)) * MLP(x) into out [T, H] bf16, scratch at ws (layout L), timeouts reported to err.
static int shared_fp8_run(const void* x, const void* w_sg, const uint8_t* w13, const float* w13_s,
                          const uint8_t* w2, const float* w2_s, int T, int H, int Is, void* out,
                          const SharedLayout& L, uint8_t* ws, int32_t* err, const DeviceInfo& d, cudaStream_t s) {
    float* gate = reinterpret_cast<float*>(ws + L.gate);
    int32_t* expert_ids = reinterpret_cast<int32_t*>(ws + L.expert_ids);
    int32_t* npp = reinterpret_cast<int32_t*>(ws + L.npp);
    uint8_t* xq = ws + L.xq;
    float* xs = reinterpret_cast<float*>(ws + L.xs);
    uint8_t* a2 = ws + L.a2;
    float* a2s = reinterpret_cast<float*>(ws + L.a2s);
    if (launch_shared_gate(x, w_sg, T, H, gate, expert_ids, npp, d.sms, s) != cudaSuccess) return PM_ERR_CUDA;
    if (launch_quant_fp8(x, T, H, 1, nullptr, xq, xs, s) != cudaSuccess) return PM_ERR_CUDA;
    CUtensorMap ta, tb;
    if (!encode_tmap_2d_u8(&ta, xq, (uint64_t)H, (uint64_t)L.rows, (uint64_t)H, 128, 128) ||
        !encode_tmap_2d_u8(&tb, w13, (uint64_t)H, (uint64_t)2 * Is, (uint64_t)H, 128, 128))
        return PM_ERR_CUDA;
    GemmArgs g1 = gemm_args_common(xs, w13_s, expert_ids, npp, 2 * Is, H, Is / 128, L.rows, Is, err);
    g1.out_q = a2;
    g1.out_s = a2s;
    if (launch_gemm_fp8(0, ta, tb, g1, d.sms, s) != cudaSuccess) return PM_ERR_CUDA;
    if (!encode_tmap_2d_u8(&ta, a2, (uint64_t)Is, (uint64_t)L.rows, (uint64_t)Is, 128, 128) ||
        !encode_tmap_2d_u8(&tb, w2, (uint64_t)Is, (uint64_t)H, (uint64_t)Is, 128, 128))
        return PM_ERR_CUDA;
    GemmArgs g2 = gemm_args_common(a2s, w2_s, expert_ids, npp, H, Is, H / 256, L.rows, Is, err);
    g2.sorted_ids = nullptr;  // row t of the block is token t
    g2.topk_w = gate;
    g2.c3 = static_cast<__nv_bfloat16*>(out);
    g2.n_valid = T;
    g2.round_first = 1;  // MLP output rounded to bf16, then the bf16 product with the bf16 gate
    return cuda_status(launch_gemm_fp8(1, ta, tb, g2, d.sms, s));
}

size_t pm_moe_shared_workspace_bytes(int T, int H, int Is) {
    if (check_shared_dims(T, H, Is) != PM_OK) return 0;
    return shared_layout_of(T, H, Is, false).total;
}

int pm_moe_shared_fp8(const void* x, const void* w_sg, const uint8_t* w13, const float* w13_s, const uint8_t* w2,
                      const float* w2_s, int T, int H, int Is, void* out, void* workspace, size_t workspace_bytes,
                      pm_stream_t stream) {
    int st = check_shared_dims(T, H, Is);
    if (st != PM_OK) return st;
    if (T == 0) return PM_OK;
    if (!x || !w_sg || !w13 || !w13_s || !w2 || !w2_s || !out || !workspace) return PM_ERR_INVALID;
    if (!a16(x) || !a16(w_sg) || !a16(w13) || !a16(w2) || !a16(out) || !a16(workspace)) return PM_ERR_ALIGN;
    const SharedLayout L = shared_layout_of(T, H, Is, false);
    if (workspace_bytes < L.total) return PM_ERR_WORKSPACE;
    DeviceInfo d;
    st = current_device_info(&d);
    if (st != PM_OK) return st;
    cudaStream_t s = (cudaStream_t)stream;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    int32_t* status = reinterpret_cast<int32_t*>(ws + L.status);
    if (cudaMemsetAsync(status, 0, 4 * sizeof(int32_t), s) != cudaSuccess) return PM_ERR_CUDA;
    return shared_fp8_run(x, w_sg, w13, w13_s, w2, w2_s, T, H, Is, out, L, ws, status, d, s);
}

size_t pm_moe_block_workspace_bytes(int T, int H, int I, int Is, int E, int k) {
    if (check_dims(T, H, I, E, k) != PM_OK || check_shared_dims(T, H, Is) != PM_OK) return 0;
    return layout_of(T, H, I, E, k, PM_FMT_FP8).total + shared_layout_of(T, H, Is, true).total;
}

int pm_moe_block_fp8(const void* x, const void* router_w, const void* logits, const uint8_t* w1, const float* w1_s,
                     const uint8_t* w2, const float* w2_s, const void* w_sg, const uint8_t* sw13,
                     const float* sw13_s, const uint8_t* sw2, const float* sw2_s, int T, int H, int I, int Is, int E,
                     int k, void* out, void* workspace, size_t workspace_bytes, pm_stream_t stream) {
    int st = check_dims(T, H, I, E, k);
    if (st != PM_OK) return st;
    st = check_shared_dims(T, H, Is);
    if (st != PM_OK) return st;
    if (T == 0) return PM_OK;
    if (!x || !out || !w_sg || !sw13 || !sw13_s || !sw2 || !sw2_s || !workspace) return PM_ERR_INVALID;
    if (!a16(x) || !a16(out) || !a16(w_sg) || !a16(sw13) || !a16(sw2) || !a16(workspace)) return PM_ERR_ALIGN;
    const size_t routed = layout_of(T, H, I, E, k, PM_FMT_FP8).total;
    const SharedLayout L = shared_layout_of(T, H, Is, true);
    if (workspace_bytes < routed + L.total) return PM_ERR_WORKSPACE;
    DeviceInfo d;
    st = current_device_info(&d);
    if (st != PM_OK) return st;
    cudaStream_t s = (cudaStream_t)stream;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    int32_t* status = reinterpret_cast<int32_t*>(ws);  // the routed layout's status region comes first
    if (cudaMemsetAsync(status, 0, 4 * sizeof(int32_t), s) != cudaSuccess) return PM_ERR_CUDA;
    uint8_t* sws = ws + routed;
    // The shared expert runs on this thread's side stream, forked from and joined back into the caller's stream
    // (events, so a graph capture records two branches): its kernels overlap the routed routing kernels, which
    // leave most SMs idle, and the final sum waits for it.
    SideStream* side = side_stream();
    if (side == nullptr) return PM_ERR_CUDA;
    if (cudaEventRecord(side->fork, s) != cudaSuccess ||
        cudaStreamWaitEvent(side->stream, side->fork, 0) != cudaSuccess)
        return PM_ERR_CUDA;
    st = shared_fp8_run(x, w_sg, sw13, sw13_s, sw2, sw2_s, T, H, Is, sws + L.out, L, sws, status, d, side->stream);
    if (st != PM_OK) return st;
    if (cudaEventRecord(side->join, side->stream) != cudaSuccess) return PM_ERR_CUDA;
    return forward_fp8_impl(x, router_w, logits, w1, w1_s, w2, w2_s, T, H, I, E, k, sws + L.out, side->join, out,
                            workspace, routed, stream, false);
}

int pm_moe_quant_nvfp4(const void* x, int T, int H, int k, const int32_t* slot_of, float gs, uint8_t* a_q,
                       uint8_t* a_sf, pm_stream_t stream) {
    if (T < 0 || H <= 0 || (slot_of != nullptr && k <= 0) || !(gs > 0.0f)) return PM_ERR_INVALID;
    if (H % 64 != 0) return PM_ERR_SHAPE;
    if (T == 0) return PM_OK;
    if (!x || !a_q || !a_sf) return PM_ERR_INVALID;
    if (!a16(x) || !a16(a_q) || !a16(a_sf)) return PM_ERR_ALIGN;
    DeviceInfo d;
    const int st = current_device_info(&d);
    if (st != PM_OK) return st;
    return cuda_status(launch_quant_nvfp4(x, T, H, k, slot_of, gs, a_q, a_sf, (cudaStream_t)stream));
}

static int check_nvfp4_dims(int T, int H, int I, int E, int k) {
    const int st = check_dims(T, H, I, E, k);
    if (st != PM_OK) return st;
    return (I % 256 == 0) ? PM_OK : PM_ERR_SHAPE;
}

int pm_moe_gemm1_nvfp4(const uint8_t* a_q, const uint8_t* a_sf, const uint8_t* w1, const uint8_t* w1_sf,
                       const float* alpha1, float a2_gs, const int32_t* expert_ids, const int32_t* num_post_pad,
                       int max_slots, int H, int I, int E, uint8_t* out_q, uint8_t* out_sf, int32_t* err,
                       pm_stream_t stream) {
    int st = check_nvfp4_dims(0, H, I, E, 1);
    if (st != PM_OK) return st;
    if (max_slots < 0 || max_slots % kBlockM != 0 || !(a2_gs > 0.0f)) return PM_ERR_SHAPE;
    if (max_slots == 0) return PM_OK;
    if (!a_q || !a_sf || !w1 || !w1_sf || !alpha1 || !expert_ids || !num_post_pad || !out_q || !out_sf)
        return PM_ERR_INVALID;
    if (!a16(a_q) || !a16(a_sf) || !a16(w1) || !a16(w1_sf) || !a16(out_q) || !a16(out_sf)) return PM_ERR_ALIGN;
    DeviceInfo d;
    st = current_device_info(&d);
    if (st != PM_OK) return st;
    CUtensorMap ta, tb;
    if (!encode_tmap_2d_u8(&ta, a_q, (uint64_t)H / 2, (uint64_t)max_slots, (uint64_t)H / 2, 128, 128) ||
        !encode_tmap_2d_u8(&tb, w1, (uint64_t)H / 2, (uint64_t)E * 2 * I, (uint64_t)H / 2, 128, 128))
        return PM_ERR_CUDA;
    NvGemmArgs g;
    memset(&g, 0, sizeof(g));
    g.a_sf = a_sf;
    g.b_sf = w1_sf;
    g.alpha = alpha1;
    g.expert_ids = expert_ids;
    g.num_post_pad = num_post_pad;
    g.n_total = 2 * I;
    g.K = H;
    g.n_tiles = I / 128;
    g.max_tiles = (max_slots / kBlockM) * g.n_tiles;
    g.inter = I;
    g.gs_out = a2_gs;
    g.out_q = out_q;
    g.out_sf = out_sf;
    g.err = err;
    return cuda_status(launch_gemm_nvfp4(0, ta, tb, g, d.sms, (cudaStream_t)stream));
}

int pm_moe_gemm2_nvfp4(const uint8_t* a_q, const uint8_t* a_sf, const uint8_t* w2, const uint8_t* w2_sf,
                       const float* alpha2, const int32_t* expert_ids, const int32_t* num_post_pad,
                       const int32_t* sorted_ids, const float* topk_w, int max_slots, int T, int k, int H, int I,
                       int E, void* c3, int32_t* err, pm_stream_t stream) {
    int st = check_nvfp4_dims(T, H, I, E, k);
    if (st != PM_OK) return st;
    if (max_slots < 0 || max_slots % kBlockM != 0) return PM_ERR_SHAPE;
    if (max_slots == 0 || T == 0) return PM_OK;
    if (!a_q || !a_sf || !w2 || !w2_sf || !alpha2 || !expert_ids || !num_post_pad || !sorted_ids || !topk_w || !c3)
        return PM_ERR_INVALID;
    if (!a16(a_q) || !a16(a_sf) || !a16(w2) || !a16(w2_sf) || !a16(c3)) return PM_ERR_ALIGN;
    DeviceInfo d;
    st = current_device_info(&d);
    if (st != PM_OK) return st;
    CUtensorMap ta, tb;
    if (!encode_tmap_2d_u8(&ta, a_q, (uint64_t)I / 2, (uint64_t)max_slots, (uint64_t)I / 2, 128, 128) ||
        !encode_tmap_2d_u8(&tb, w2, (uint64_t)I / 2, (uint64_t)E * H, (uint64_t)I / 2, 128, 128))
        return PM_ERR_CUDA;
    NvGemmArgs g;
    memset(&g, 0, sizeof(g));
    g.a_sf = a_sf;
    g.b_sf = w2_sf;
    g.alpha = alpha2;
    g.expert_ids = expert_ids;
    g.num_post_pad = num_post_pad;
    g.n_total = H;
    g.K = I;
    g.n_tiles = H / 256;
    g.max_tiles = (max_slots / kBlockM) * g.n_tiles;
    g.inter = I;
    g.sorted_ids = sorted_ids;
    g.topk_w = topk_w;
    g.c3 = static_cast<__nv_bfloat16*>(c3);
    g.n_valid = T * k;
    g.err = err;
    return cuda_status(launch_gemm_nvfp4(1, ta, tb, g, d.sms, (cudaStream_t)stream));
}

int pm_moe_forward_nvfp4(const void* x, const void* router_w, const void* logits, const uint8_t* w1,
                         const uint8_t* w1_sf, const float* alpha1, float a1_gs, const uint8_t* w2,
                         const uint8_t* w2_sf, const float* alpha2, float a2_gs, int T, int H, int I, int E, int k,
                         void* out, void* workspace, size_t workspace_bytes, pm_stream_t stream) {
    int st = check_nvfp4_dims(T, H, I, E, k);
    if (st != PM_OK) return st;
    if (T == 0) return PM_OK;
    if (!x || !w1 || !w1_sf || !alpha1 || !w2 || !w2_sf || !alpha2 || !out || !workspace || (!router_w && !logits))
        return PM_ERR_INVALID;
    if (!(a1_gs > 0.0f) || !(a2_gs > 0.0f)) return PM_ERR_INVALID;
    if (!a16(x) || !a16(w1) || !a16(w2) || !a16(out) || !a16(workspace) || (router_w && !logits && !a16(router_w)))
        return PM_ERR_ALIGN;
    const Layout L = layout_of(T, H, I, E, k, PM_FMT_NVFP4);
    if (workspace_bytes < L.total) return PM_ERR_WORKSPACE;
    DeviceInfo d;
    st = current_device_info(&d);
    if (st != PM_OK) return st;
    cudaStream_t s = (cudaStream_t)stream;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    auto R = [&](int r) { return ws + L.off[r]; };
    float* router_part = L.len[PM_WS_ROUTER_PART] > 0 ? reinterpret_cast<float*>(R(PM_WS_ROUTER_PART)) : nullptr;
    int32_t* status = reinterpret_cast<int32_t*>(R(PM_WS_STATUS));
    float* topk_w = reinterpret_cast<float*>(R(PM_WS_TOPK_W));
    int32_t* topk_ids = reinterpret_cast<int32_t*>(R(PM_WS_TOPK_IDS));
    int32_t* sorted = reinterpret_cast<int32_t*>(R(PM_WS_SORTED));
    int32_t* expert_ids = reinterpret_cast<int32_t*>(R(PM_WS_EXPERT_IDS));
    int32_t* npp = reinterpret_cast<int32_t*>(R(PM_WS_NUM_POST_PAD));
    int32_t* slot_of = reinterpret_cast<int32_t*>(R(PM_WS_SLOT_OF));
    // the status words start at zero: zeroed by the router kernel when it runs (no memset between this forward's
    // first kernel and the previous one's last), else by a memset
    if (logits != nullptr && cudaMemsetAsync(status, 0, L.len[PM_WS_STATUS], s) != cudaSuccess) return PM_ERR_CUDA;
    cudaError_t e =
        logits != nullptr
            ? launch_topk(logits, nullptr, T, E, k, topk_w, topk_ids, s)
            : launch_router_topk(x, router_w, nullptr, T, H, E, k, R(PM_WS_LOGITS), topk_w, topk_ids, status, s,
                                 router_part, true, status);
    if (e != cudaSuccess) return PM_ERR_CUDA;
    e = launch_align(topk_ids, T * k, E, reinterpret_cast<int32_t*>(R(PM_WS_COUNTS)), sorted, expert_ids, npp,
                     reinterpret_cast<int32_t*>(R(PM_WS_EXPERT_OFF)), slot_of, s);
    if (e != cudaSuccess) return PM_ERR_CUDA;
    e = launch_quant_nvfp4(x, T, H, k, slot_of, a1_gs, R(PM_WS_A1), R(PM_WS_A1_SCALE), s);
    if (e != cudaSuccess) return PM_ERR_CUDA;
    st = pm_moe_gemm1_nvfp4(R(PM_WS_A1), R(PM_WS_A1_SCALE), w1, w1_sf, alpha1, a2_gs, expert_ids, npp, L.max_slots,
                            H, I, E, R(PM_WS_A2), R(PM_WS_A2_SCALE), status, stream);
    if (st != PM_OK) return st;
    st = pm_moe_gemm2_nvfp4(R(PM_WS_A2), R(PM_WS_A2_SCALE), w2, w2_sf, alpha2, expert_ids, npp, sorted, topk_w,
                            L.max_slots, T, k, H, I, E, R(PM_WS_C3), status, stream);
    if (st != PM_OK) return st;
    return cuda_status(launch_combine(R(PM_WS_C3), nullptr, T, k, H, out, s));
}

// ------------------------------------------------------------------------------------------- dense projection
struct DenseLayout {
    size_t status, ones, expert_ids, npp, xq, xs, total;
    int rows;
};

static DenseLayout dense_layout_of(int T, int K) {
    DenseLayout L;
    const int rows = (T + kBlockM - 1) / kBlockM * kBlockM;
    size_t o = 0;
    auto take = [&](size_t bytes) { const size_t at = o; o = align256(o + bytes); return at; };
    L.status = take(4 * sizeof(int32_t));
    L.ones = take((size_t)T * 4);
    L.expert_ids = take((size_t)(rows / kBlockM) * 4);
    L.npp = take(4);
    L.xq = take((size_t)rows * K);
    L.xs = take((size_t)rows * (K / 128) * 4);
    L.total = o;
    L.rows = rows;
    return L;
}

static int check_dense_dims(int T, int K, int N) {
    if (T < 0 || K <= 0 || N <= 0) return PM_ERR_INVALID;
    if (K % 128 != 0 || N % 256 != 0 || (long)T * (K > N ? K : N) > (1L << 34) || T > (1 << 30))
        return PM_ERR_SHAPE;
    return PM_OK;
}

size_t pm_fp8_linear_workspace_bytes(int T, int K, int N) {
    if (check_dense_dims(T, K, N) != PM_OK) return 0;
    return dense_layout_of(T, K).total;
}

int pm_fp8_linear(const void* x, const uint8_t* w, const float* w_s, int T, int K, int N, void* out,
                  void* workspace, size_t workspace_bytes, pm_stream_t stream) {
    int st = check_dense_dims(T, K, N);
    if (st != PM_OK) return st;
    if (T == 0) return PM_OK;
    if (!x || !w || !w_s || !out || !workspace) return PM_ERR_INVALID;
    if (!a16(x) || !a16(w) || !a16(out) || !a16(workspace)) return PM_ERR_ALIGN;
    const DenseLayout L = dense_layout_of(T, K);
    if (workspace_bytes < L.total) return PM_ERR_WORKSPACE;
    DeviceInfo d;
    st = current_device_info(&d);
    if (st != PM_OK) return st;
    cudaStream_t s = (cudaStream_t)stream;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    int32_t* status = reinterpret_cast<int32_t*>(ws + L.status);
    float* ones = reinterpret_cast<float*>(ws + L.ones);
    int32_t* expert_ids = reinterpret_cast<int32_t*>(ws + L.expert_ids);
    int32_t* npp = reinterpret_cast<int32_t*>(ws + L.npp);
    uint8_t* xq = ws + L.xq;
    float* xs = reinterpret_cast<float*>(ws + L.xs);
    if (cudaMemsetAsync(status, 0, 4 * sizeof(int32_t), s) != cudaSuccess) return PM_ERR_CUDA;
    if (launch_dense_plan(T, ones, expert_ids, npp, d.sms, s) != cudaSuccess) return PM_ERR_CUDA;
    if (launch_quant_fp8(x, T, K, 1, nullptr, xq, xs, s) != cudaSuccess) return PM_ERR_CUDA;
    CUtensorMap ta, tb;
    if (!encode_tmap_2d_u8(&ta, xq, (uint64_t)K, (uint64_t)L.rows, (uint64_t)K, 128, 128) ||
        !encode_tmap_2d_u8(&tb, w, (uint64_t)K, (uint64_t)N, (uint64_t)K, 128, 128))
        return PM_ERR_CUDA;
    GemmArgs g = gemm_args_common(xs, w_s, expert_ids, npp, N, K, N / 256, L.rows, K, status);
    g.sorted_ids = nullptr;  // row t is token t
    g.topk_w = ones;
    g.c3 = static_cast<__nv_bfloat16*>(out);
    g.n_valid = T;
    return cuda_status(launch_gemm_fp8(1, ta, tb, g, d.sms, s));
}

static int nvfp4_prepare_impl(const uint8_t* w, const float* s, int E, int R, int C, uint8_t* packed,
                              uint8_t* scales, float* g, pm_stream_t stream, bool search, const float* imp) {
    if (E < 0 || R < 0 || C < 0) return PM_ERR_INVALID;
    if (R % 128 != 0 || C % 128 != 0 || (long)E * R > (1L << 31) || (long)E * R * C / 16 > (1L << 31))
        return PM_ERR_SHAPE;
    if (E == 0 || R == 0 || C == 0) return PM_OK;
    if (!w || !s || !packed || !scales || !g) return PM_ERR_INVALID;
    if (!a16(w) || (reinterpret_cast<uintptr_t>(packed) & 7u) != 0 || (reinterpret_cast<uintptr_t>(s) & 3u) != 0 ||
        (reinterpret_cast<uintptr_t>(g) & 3u) != 0)
        return PM_ERR_ALIGN;
    DeviceInfo d;
    const int st = current_device_info(&d);
    if (st != PM_OK) return st;
    if (imp != nullptr && !a16(imp)) return PM_ERR_ALIGN;
    return cuda_status(
        launch_nvfp4_prepare(w, s, E, R, C, packed, scales, g, d.sms, (cudaStream_t)stream, search, imp));
}

int pm_nvfp4_prepare(const uint8_t* w, const float* s, int E, int R, int C, uint8_t* packed, uint8_t* scales,
                     float* g, pm_stream_t stream) {
    return nvfp4_prepare_impl(w, s, E, R, C, packed, scales, g, stream, false, nullptr);
}

int pm_nvfp4_prepare_search(const uint8_t* w, const float* s, const float* importance, int E, int R, int C,
                            uint8_t* packed, uint8_t* scales, float* g, pm_stream_t stream) {
    return nvfp4_prepare_impl(w, s, E, R, C, packed, scales, g, stream, true, importance);
}

// ---------------------------------------------------------------------------------------- expert parallelism
int pm_ep_alloc(size_t bytes, void** ptr, void* ipc_handle) {
    if (!ptr || !ipc_handle || bytes == 0) return PM_ERR_INVALID;
    DeviceInfo d;
    const int st = current_device_info(&d);
    if (st != PM_OK) return st;
    void* p = nullptr;
    if (cudaMalloc(&p, bytes) != cudaSuccess) return PM_ERR_CUDA;
    cudaIpcMemHandle_t h;
    if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
        cudaFree(p);
        return PM_ERR_CUDA;
    }
    memcpy(ipc_handle, &h, sizeof(h));
    *ptr = p;
    return PM_OK;
}

int pm_ep_open(const void* ipc_handle, void** ptr) {
    if (!ptr || !ipc_handle) return PM_ERR_INVALID;
    cudaIpcMemHandle_t h;
    memcpy(&h, ipc_handle, sizeof(h));
    return cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess ? PM_OK : PM_ERR_CUDA;
}

int pm_ep_close(void* ptr) { return ptr && cudaIpcCloseMemHandle(ptr) == cudaSuccess ? PM_OK : PM_ERR_CUDA; }

int pm_ep_free(void* ptr) { return ptr && cudaFree(ptr) == cudaSuccess ? PM_OK : PM_ERR_CUDA; }

int pm_ep_count(const int32_t* ids, int n, int E, int G, int rank, const uint64_t* peer_cm, pm_stream_t stream) {
    if (n < 0 || E <= 0 || E > kMaxExperts || G <= 0 || rank < 0 || rank >= G) return PM_ERR_INVALID;
    if ((n > 0 && !ids) || !peer_cm) return PM_ERR_INVALID;
    return cuda_status(launch_ep_count(ids, n, E, G, rank, peer_cm, (cudaStream_t)stream));
}

int pm_ep_barrier(const uint64_t* peer_flag, unsigned* own_flag, int G, unsigned target, int32_t* err,
                  uint64_t wait_limit_ns, pm_stream_t stream) {
    if (!peer_flag || !own_flag || G <= 0) return PM_ERR_INVALID;
    return cuda_status(launch_ep_barrier(peer_flag, own_flag, G, target, err, wait_limit_ns, (cudaStream_t)stream));
}

int pm_ep_offsets(const int32_t* cm, int G, int E, int epr, int rank, int32_t* base, int32_t* expert_ids,
                  int32_t* num_post_pad, int cap_slots, int32_t* err, int32_t* bounds, int groups,
                  pm_stream_t stream) {
    if (!cm || !base || !expert_ids || !num_post_pad || !err || G <= 0 || epr <= 0 || E != G * epr ||
        E > kMaxExperts || rank < 0 || rank >= G || cap_slots % kBlockM != 0)
        return PM_ERR_INVALID;
    if (bounds != nullptr && (groups < 1 || epr % groups != 0)) return PM_ERR_INVALID;
    return cuda_status(launch_ep_offsets(cm, G, E, epr, rank, base, expert_ids, num_post_pad, cap_slots / kBlockM,
                                         err, bounds, groups, (cudaStream_t)stream));
}

int pm_ep_dispatch_quant(const void* x, int T, int H, int k, const int32_t* topk_ids, const float* topk_w,
                         const int32_t* slot_local, const int32_t* expert_off_local, const int32_t* base, int E,
                         int epr, int rank, int cap_slots, const uint64_t* peer_a1, const uint64_t* peer_a1_scale,
                         const uint64_t* peer_meta, const uint64_t* peer_weight, int32_t* err, int local_lo,
                         int local_hi, int max_sms, pm_stream_t stream) {
    if (T < 0 || H <= 0 || H % 128 != 0 || k <= 0 || epr <= 0 || E <= 0 || rank < 0 || cap_slots <= 0 ||
        local_lo < 0 || local_hi > epr || local_lo >= local_hi || max_sms < 0)
        return PM_ERR_INVALID;
    if ((long)T * k >= (1L << 24) || rank >= 128) return PM_ERR_TOO_LARGE;
    if (T == 0) return PM_OK;
    if (!x || !topk_ids || !topk_w || !slot_local || !expert_off_local || !base || !peer_a1 || !peer_a1_scale ||
        !peer_meta || !peer_weight || !err)
        return PM_ERR_INVALID;
    if (!a16(x)) return PM_ERR_ALIGN;
    DeviceInfo d;
    const int st = current_device_info(&d);
    if (st != PM_OK) return st;
    // max_sms: one 1024-thread CTA per SM left free beside a GEMM; 0: the whole GPU
    const int ctas = max_sms > 0 && max_sms < d.sms ? max_sms : 0;
    return cuda_status(launch_ep_dispatch_quant(x, T, H, k, topk_ids, topk_w, slot_local, expert_off_local, base, E,
                                                epr, rank, cap_slots, peer_a1, peer_a1_scale, peer_meta, peer_weight,
                                                err, d.sms, local_lo, local_hi, ctas, (cudaStream_t)stream));
}

int pm_ep_local_rows(const int32_t* meta, const int32_t* num_post_pad, int cap_slots, int H, int G, int n_pairs,
                     const uint64_t* peer_back, uint64_t* dst_rows, int32_t* err, pm_stream_t stream) {
    if (!meta || !num_post_pad || !peer_back || !dst_rows || !err || cap_slots <= 0 || H <= 0 || G <= 0)
        return PM_ERR_INVALID;
    DeviceInfo d;
    const int st = current_device_info(&d);
    if (st != PM_OK) return st;
    return cuda_status(launch_ep_local_rows(meta, num_post_pad, cap_slots, H, G, n_pairs, peer_back, dst_rows, err,
                                            d.sms, (cudaStream_t)stream));
}

int pm_ep_gemm1_fp8(const uint8_t* a_q, const float* a_s, const uint8_t* w1, const float* w1_s,
                    const int32_t* expert_ids, const int32_t* bounds, int group, int cap_slots, int H, int I, int E,
                    uint8_t* out_q, float* out_s, int32_t* err, int max_sms, pm_stream_t stream) {
    int st = check_dims(1, H, I, E, 1);
    if (st != PM_OK) return st;
    if (cap_slots <= 0 || cap_slots % kBlockM != 0 || group < 0 || max_sms < 0) return PM_ERR_SHAPE;
    if (!a_q || !a_s || !w1 || !w1_s || !expert_ids || !bounds || !out_q || !out_s) return PM_ERR_INVALID;
    if (!a16(a_q) || !a16(w1) || !a16(out_q)) return PM_ERR_ALIGN;
    DeviceInfo d;
    st = current_device_info(&d);
    if (st != PM_OK) return st;
    CUtensorMap ta, tb;
    if (!encode_tmap_2d_u8(&ta, a_q, (uint64_t)H, (uint64_t)cap_slots, (uint64_t)H, 128, 128) ||
        !encode_tmap_2d_u8(&tb, w1, (uint64_t)H, (uint64_t)E * 2 * I, (uint64_t)H, 128, 128))
        return PM_ERR_CUDA;
    // slots [bounds[group], bounds[group + 1]): the GEMM starts at the first and ends at the second
    GemmArgs g = gemm_args_common(a_s, w1_s, expert_ids, bounds + group + 1, 2 * I, H, I / 128, cap_slots, I, err);
    g.slot_lo = bounds + group;
    g.out_q = out_q;
    g.out_s = out_s;
    const int sms = max_sms > 0 && max_sms < d.sms ? max_sms : d.sms;
    return cuda_status(launch_gemm_fp8(0, ta, tb, g, sms, (cudaStream_t)stream));
}

int pm_ep_gemm2_fp8(const uint8_t* a_q, const float* a_s, const uint8_t* w2, const float* w2_s,
                    const int32_t* expert_ids, const int32_t* num_post_pad, const float* weight,
                    const uint64_t* dst_rows, int cap_slots, int H, int I, int E, int32_t* err, pm_stream_t stream) {
    int st = check_dims(1, H, I, E, 1);
    if (st != PM_OK) return st;
    if (cap_slots <= 0 || cap_slots % kBlockM != 0) return PM_ERR_SHAPE;
    if (!a_q || !a_s || !w2 || !w2_s || !expert_ids || !num_post_pad || !weight || !dst_rows) return PM_ERR_INVALID;
    if (!a16(a_q) || !a16(w2)) return PM_ERR_ALIGN;
    DeviceInfo d;
    st = current_device_info(&d);
    if (st != PM_OK) return st;
    CUtensorMap ta, tb;
    if (!encode_tmap_2d_u8(&ta, a_q, (uint64_t)I, (uint64_t)cap_slots, (uint64_t)I, 128, 128) ||
        !encode_tmap_2d_u8(&tb, w2, (uint64_t)I, (uint64_t)E * H, (uint64_t)I, 128, 128))
        return PM_ERR_CUDA;
    GemmArgs g = gemm_args_common(a_s, w2_s, expert_ids, num_post_pad, H, I, H / 256, cap_slots, I, err);
    g.sorted_ids = nullptr;  // the slot is the row: weight[slot], destination dst_rows[slot]
    g.topk_w = weight;
    g.dst_rows = dst_rows;
    g.n_valid = cap_slots;
    return cuda_status(launch_gemm_fp8(1, ta, tb, g, d.sms, (cudaStream_t)stream));
}

int pm_moe_read_status(const void* workspace, pm_stream_t stream) {
    if (!workspace) return PM_ERR_INVALID;
    int32_t flag = 0;
    if (cudaMemcpyAsync(&flag, workspace, sizeof(flag), cudaMemcpyDeviceToHost, (cudaStream_t)stream) != cudaSuccess)
        return PM_ERR_CUDA;
    if (cudaStreamSynchronize((cudaStream_t)stream) != cudaSuccess) return PM_ERR_CUDA;
    return flag ? PM_ERR_TIMEOUT : PM_OK;
}

}  // extern "C"
