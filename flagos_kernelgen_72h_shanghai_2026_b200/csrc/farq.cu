// farq.cu — host side of libfarq.so: argument validation, launch planning
// and the C ABI declared in include/farq.h. Device code: farq_kernel.cuh,
// instantiated in farq_inst_*.cu.
//
// The reference picks one of three Triton kernels per call from a backend
// tag and (M, D) (src/task01_fused_add_rmsnorm_group_quant.py:1731-1851);
// here the host picks the template parameters (vectors per thread K, group
// lanes G/8) and the launch shape (team size, teams per CTA, pipeline
// stages, grid) of one kernel.
#include <cuda_runtime.h>
#include <stdint.h>
#include <atomic>

#include "farq.h"
#include "farq_kernel.cuh"
#include "farq_ar_kernel.cuh"

namespace farq {

constexpr int kMaxDevices = 64;
constexpr int kSlots = 2 * 2 * kMaxK * 6;
std::atomic<int> g_sm_count[kMaxDevices];
std::atomic<int> g_smem_optin[kMaxDevices];
std::atomic<int> g_smem_set[kMaxDevices][kSlots];  // largest dynamic smem granted
std::atomic<int> g_regs[kMaxDevices][kSlots];      // registers per thread (0 = unknown)
std::atomic<int> g_ar_smem_set[kMaxDevices][kSlots * 4];  // same, tensor-parallel kernels
std::atomic<int> g_ar_regs[kMaxDevices][kSlots * 4];      // (x4: WMAX 1, 2, 4, 8)

int ilog2(int v) {
  int l = 0;
  while ((1 << l) < v) ++l;
  return l;
}

struct KernelSel {
  KernelFn fn;
  int slot;
};
KernelSel select_kernel(int x_dtype, bool e4m3, int K, int G) {
  const int gl = ilog2(G / 8);
  KernelFn fn;
  if (x_dtype == FARQ_DTYPE_BF16)
    fn = e4m3 ? kernel_bf16_e4m3(K, gl) : kernel_bf16_int8(K, gl);
  else
    fn = e4m3 ? kernel_fp16_e4m3(K, gl) : kernel_fp16_int8(K, gl);
  const int slot = (((x_dtype == FARQ_DTYPE_BF16 ? 0 : 1) * 2 + (e4m3 ? 1 : 0)) * kMaxK + (K - 1)) * 6 + gl;
  return {fn, slot};
}

cudaError_t device_info(int* dev, int* sms, int* smem_optin) {
  cudaError_t e = cudaGetDevice(dev);
  if (e != cudaSuccess) return e;
  if (*dev < 0 || *dev >= kMaxDevices) return cudaErrorInvalidDevice;
  int s = g_sm_count[*dev].load(std::memory_order_relaxed);
  int o = g_smem_optin[*dev].load(std::memory_order_relaxed);
  if (s <= 0 || o <= 0) {
    e = cudaDeviceGetAttribute(&s, cudaDevAttrMultiProcessorCount, *dev);
    if (e != cudaSuccess) return e;
    e = cudaDeviceGetAttribute(&o, cudaDevAttrMaxSharedMemoryPerBlockOptin, *dev);
    if (e != cudaSuccess) return e;
    g_sm_count[*dev].store(s, std::memory_order_relaxed);
    g_smem_optin[*dev].store(o, std::memory_order_relaxed);
  }
  *sms = s;
  *smem_optin = o;
  return cudaSuccess;
}

cudaError_t kernel_regs(int dev, const KernelSel& k, int* regs) {
  int r = g_regs[dev][k.slot].load(std::memory_order_relaxed);
  if (r <= 0) {
    cudaFuncAttributes fa;
    cudaError_t e = cudaFuncGetAttributes(&fa, reinterpret_cast<const void*>(k.fn));
    if (e != cudaSuccess) return e;
    r = fa.numRegs;
    g_regs[dev][k.slot].store(r, std::memory_order_relaxed);
  }
  *regs = r;
  return cudaSuccess;
}

int dtype_size(int dt) {
  switch (dt) {
    case FARQ_DTYPE_BF16:
    case FARQ_DTYPE_FP16: return 2;
    case FARQ_DTYPE_FP32: return 4;
    case FARQ_DTYPE_INT8:
    case FARQ_DTYPE_E4M3: return 1;
    default: return 0;
  }
}
bool is_float_out(int dt) {
  return dt == FARQ_DTYPE_BF16 || dt == FARQ_DTYPE_FP16 || dt == FARQ_DTYPE_FP32;
}

struct Tune {
  int ctas_per_sm, teams, stages, k;
};
struct Plan {
  int team_threads, teams, K, grid, stages;
  size_t smem;
};

// Shared memory of one SM (B200: 228 KB) and the per-CTA system reserve.
constexpr int kSmemPerSm = 228 * 1024;
constexpr int kSmemReservedPerCta = 1024;
constexpr int kRegsPerSm = 65536;

// Vectors per thread K and team size T for a row of nvec 16-byte vectors.
// When every row gets an SM of its own (M <= #SMs, latency-bound), the widest
// team (up to 512 threads) finishes a row soonest: 1 x 7168 in 3.6 us instead
// of 5.1 us with 128 threads. Otherwise teams of 4 warps while K <= 8 covers
// the row (more teams per SM), wider teams beyond that.
int pick_k(int64_t nvec, int tune_k, bool row_per_sm, int* K_out, int* T_out) {
  int K = tune_k > 0 ? tune_k
                     : (int)(row_per_sm ? (nvec + kMaxTeamThreads - 1) / kMaxTeamThreads
                                        : (nvec + 127) / 128);
  if (K < 1) K = 1;
  if (K > kMaxK) K = kMaxK;
  const int64_t per = (nvec + K - 1) / K;
  const int64_t T = (per + 31) / 32 * 32;
  if (T > kMaxTeamThreads) return FARQ_ERR_UNSUPPORTED;
  *K_out = K;
  *T_out = (int)T;
  return FARQ_OK;
}

int make_plan(int64_t M, int64_t D, int x_dtype, int sms, int smem_optin, int regs, int K, int T,
              const Tune& tune, Plan* pl) {
  const uint32_t row_bytes = (uint32_t)(D * dtype_size(x_dtype));
  const int ctas = tune.ctas_per_sm > 0 ? tune.ctas_per_sm : 1;
  int64_t smem_cap = kSmemPerSm / ctas - kSmemReservedPerCta;
  if (smem_cap > smem_optin) smem_cap = smem_optin;
  const int regs_alloc = (regs + 7) / 8 * 8;
  int teams_cap = kMaxCtaThreads / T;
  const int by_regs = kRegsPerSm / (ctas * T * regs_alloc);
  if (by_regs < teams_cap) teams_cap = by_regs;
  if (teams_cap > kMaxTeams) teams_cap = kMaxTeams;
  if (teams_cap < 1) teams_cap = 1;
  auto fits = [&](int teams, int stages) {
    return (int64_t)smem_layout((int)D, row_bytes, teams, stages).total <= smem_cap;
  };
  // Ring slots that fit next to gamma (at most kMaxStages).
  auto max_slots = [&](int teams) {
    int s = kMaxStages;
    while (s > 0 && !fits(teams, s)) --s;
    return s;
  };
  int teams = teams_cap;
  if (tune.teams > 0 && tune.teams < teams) teams = tune.teams;
  // Small M: spread rows over SMs before stacking teams on one SM.
  const int64_t per_sm = (M + (int64_t)sms * ctas - 1) / ((int64_t)sms * ctas);
  if (per_sm < teams) teams = (int)(per_sm < 1 ? 1 : per_sm);
  // Every team needs a slot of its own (S >= teams).
  while (teams > 1 && max_slots(teams) < teams) --teams;
  // Default ring: one slot per team. More slots keep more rows in flight but
  // measured slower on B200 (4 teams: 4 slots 39.7 us, 7 slots 42.9 us at
  // 4096 x 7168), so extra slots are opt-in through tune.stages.
  int stages = max_slots(teams);
  if (stages > teams) stages = teams;
  const int slots_fit = max_slots(teams);
  if (tune.stages > 0)  // requested ring slots, clamped to [teams, what fits]
    stages = tune.stages < teams ? teams : (tune.stages < slots_fit ? tune.stages : slots_fit);
  if (stages < 1 || stages < teams) return FARQ_ERR_UNSUPPORTED;
  int64_t grid = (M + teams - 1) / teams;
  if (grid > (int64_t)sms * ctas) grid = (int64_t)sms * ctas;
  if (grid < 1) grid = 1;
  pl->team_threads = T;
  pl->teams = teams;
  pl->K = K;
  pl->grid = (int)grid;
  pl->stages = stages;
  pl->smem = smem_layout((int)D, row_bytes, teams, stages).total;
  return FARQ_OK;
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

int check_shape(int64_t M, int64_t D, int G) {
  if (M < 0 || D <= 0 || D % 8 != 0) return FARQ_ERR_BAD_SHAPE;
  if (G < 8 || G > 256 || (G & (G - 1)) != 0) return FARQ_ERR_BAD_GROUP;
  if (D % G != 0) return FARQ_ERR_BAD_SHAPE;
  if (D > kMaxHidden) return FARQ_ERR_UNSUPPORTED;
  return FARQ_OK;
}

// Checks of a farq_args_t that need no pointer and no device: struct size,
// reserved field, shape, group size and dtypes. Shared by farq_launch and
// farq_launch_host_noalloc (which must reject a call before it queues any
// copy).
int validate_args(const farq_args_t* a) {
  if (!a) return FARQ_ERR_NULL_POINTER;
  if (a->struct_size != sizeof(farq_args_t) || a->reserved0 != 0) return FARQ_ERR_BAD_ARGS_SIZE;
  int st = check_shape(a->M, a->D, a->group_size);
  if (st != FARQ_OK) return st;
  if (a->x_dtype != FARQ_DTYPE_BF16 && a->x_dtype != FARQ_DTYPE_FP16) return FARQ_ERR_BAD_DTYPE;
  if (!is_float_out(a->gamma_dtype) || !is_float_out(a->residual_out_dtype))
    return FARQ_ERR_BAD_DTYPE;
  if (a->norm_out && !is_float_out(a->norm_out_dtype)) return FARQ_ERR_BAD_DTYPE;
  if (a->q_dtype != FARQ_DTYPE_INT8 && a->q_dtype != FARQ_DTYPE_E4M3) return FARQ_ERR_BAD_DTYPE;
  return FARQ_OK;
}

// Plan for a validated shape on the current device.
int plan_for(int64_t M, int64_t D, int G, int x_dtype, bool e4m3, const Tune& tune, int* dev,
             KernelSel* ks, Plan* pl) {
  int sms, optin;
  if (device_info(dev, &sms, &optin) != cudaSuccess) return FARQ_ERR_CUDA;
  int K, T;
  const int ctas = tune.ctas_per_sm > 0 ? tune.ctas_per_sm : 1;
  int st = pick_k(D / 8, tune.k, M <= (int64_t)sms * ctas, &K, &T);
  if (st != FARQ_OK) return st;
  *ks = select_kernel(x_dtype, e4m3, K, G);
  int regs;
  if (kernel_regs(*dev, *ks, &regs) != cudaSuccess) return FARQ_ERR_CUDA;
  return make_plan(M, D, x_dtype, sms, optin, regs, K, T, tune, pl);
}

}  // namespace farq

using namespace farq;

extern "C" {

int farq_abi_version(void) { return FARQ_ABI_VERSION; }

int64_t farq_max_hidden(void) { return kMaxHidden; }

const char* farq_strerror(int status) {
  switch (status) {
    case FARQ_OK: return "ok";
    case FARQ_ERR_NULL_POINTER: return "a required pointer is NULL";
    case FARQ_ERR_BAD_SHAPE: return "bad shape: need M >= 0, D > 0, D % 8 == 0 and D % group_size == 0";
    case FARQ_ERR_BAD_GROUP: return "group_size must be a power of two in [8, 256]";
    case FARQ_ERR_BAD_DTYPE: return "unsupported dtype combination";
    case FARQ_ERR_ALIGNMENT: return "misaligned pointer or row stride (16-byte rows required)";
    case FARQ_ERR_UNSUPPORTED: return "hidden size or tuning choice outside the supported range (D <= 16384)";
    case FARQ_ERR_CUDA: return "a CUDA runtime call failed";
    case FARQ_ERR_BAD_ARGS_SIZE:
      return "argument struct size mismatch (header and library differ) or reserved field not 0";
    case FARQ_ERR_DEVICE_TIMEOUT: return "a bounded device-side wait ran out";
    case FARQ_ERR_NOALLOC_TOO_LARGE:
      return "call needs more than the 64 MiB staging array of farq_launch_host_noalloc; split the rows";
    default: return "unknown farq status";
  }
}

int farq_plan(int64_t M, int64_t D, int32_t group_size, int32_t x_dtype, int32_t tune_ctas_per_sm,
              int32_t tune_teams_per_cta, int32_t tune_stages, int32_t tune_vec_per_thread,
              int64_t out[6]) {
  if (!out) return FARQ_ERR_NULL_POINTER;
  int st = check_shape(M, D, group_size);
  if (st != FARQ_OK) return st;
  if (x_dtype != FARQ_DTYPE_BF16 && x_dtype != FARQ_DTYPE_FP16) return FARQ_ERR_BAD_DTYPE;
  Tune tune{tune_ctas_per_sm, tune_teams_per_cta, tune_stages, tune_vec_per_thread};
  int dev;
  KernelSel ks;
  Plan pl;
  st = plan_for(M > 0 ? M : 1, D, group_size, x_dtype, true, tune, &dev, &ks, &pl);
  if (st != FARQ_OK) return st;
  out[0] = pl.team_threads;
  out[1] = pl.teams;
  out[2] = pl.K;
  out[3] = pl.grid;
  out[4] = pl.stages;
  out[5] = (int64_t)pl.smem;
  return FARQ_OK;
}

int farq_launch(const farq_args_t* a, void* stream) {
  int st = validate_args(a);
  if (st != FARQ_OK) return st;
  const int64_t M = a->M, D = a->D;
  const int G = a->group_size;
  if (M == 0) return FARQ_OK;
  if (!a->x || !a->residual || !a->gamma || !a->residual_out || !a->x_q || !a->x_scale)
    return FARQ_ERR_NULL_POINTER;

  const int xs = dtype_size(a->x_dtype);
  const int ros = dtype_size(a->residual_out_dtype);
  const int nos = a->norm_out ? dtype_size(a->norm_out_dtype) : 0;
  const int64_t sx = a->x_row_stride ? a->x_row_stride : D;
  const int64_t sr = a->residual_row_stride ? a->residual_row_stride : D;
  const int64_t sro = a->residual_out_row_stride ? a->residual_out_row_stride : D;
  const int64_t sno = a->norm_out_row_stride ? a->norm_out_row_stride : D;
  const int64_t sq = a->x_q_row_stride ? a->x_q_row_stride : D;
  // x_scale: [M, D/G] row-major (row stride >= D/G), or with
  // FARQ_FLAG_SCALE_COLUMN_MAJOR [D/G, ld] (ld = x_scale_row_stride >= M).
  const bool scale_cm = (a->flags & FARQ_FLAG_SCALE_COLUMN_MAJOR) != 0;
  const int64_t sld = a->x_scale_row_stride ? a->x_scale_row_stride : (scale_cm ? M : D / G);
  if (sx < D || sr < D || sro < D || sq < D || (a->norm_out && sno < D) ||
      sld < (scale_cm ? M : D / G))
    return FARQ_ERR_BAD_SHAPE;
  const int64_t ss = scale_cm ? 1 : sld;    // floats between consecutive rows' scales
  const int64_t sgs = scale_cm ? sld : 1;   // floats between consecutive groups' scales
  // 16-byte rows for the bulk copies and vector stores; 8-byte q rows.
  if (!aligned(a->x, 16) || !aligned(a->residual, 16) || !aligned(a->residual_out, 16) ||
      !aligned(a->gamma, 16) || (a->norm_out && !aligned(a->norm_out, 16)) ||
      !aligned(a->x_q, 8) || !aligned(a->x_scale, 4))
    return FARQ_ERR_ALIGNMENT;
  if ((sx * xs) % 16 || (sr * xs) % 16 || (sro * ros) % 16 || (a->norm_out && (sno * nos) % 16) ||
      sq % 8)
    return FARQ_ERR_ALIGNMENT;

  const bool e4m3 = a->q_dtype == FARQ_DTYPE_E4M3;
  Tune tune{a->tune_ctas_per_sm, a->tune_teams_per_cta, a->tune_stages, a->tune_vec_per_thread};
  int dev;
  KernelSel ks;
  Plan pl;
  st = plan_for(M, D, G, a->x_dtype, e4m3, tune, &dev, &ks, &pl);
  if (st != FARQ_OK) return st;
  if ((int)pl.smem > g_smem_set[dev][ks.slot].load(std::memory_order_relaxed)) {
    if (cudaFuncSetAttribute(reinterpret_cast<const void*>(ks.fn),
                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.smem) != cudaSuccess)
      return FARQ_ERR_CUDA;
    g_smem_set[dev][ks.slot].store((int)pl.smem, std::memory_order_relaxed);
  }

  Params p;
  p.x = static_cast<const uint8_t*>(a->x);
  p.res = static_cast<const uint8_t*>(a->residual);
  p.gamma = a->gamma;
  p.rout = static_cast<uint8_t*>(a->residual_out);
  p.nout = static_cast<uint8_t*>(a->norm_out);
  p.q = static_cast<uint8_t*>(a->x_q);
  p.scale = a->x_scale;
  p.status = a->status;
  p.M = M;
  p.sx = sx * xs;
  p.sr = sr * xs;
  p.sro = sro * ros;
  p.sno = a->norm_out ? sno * nos : 0;
  p.sq = sq;
  p.ss = ss;
  p.sgs = sgs;
  p.D = (int32_t)D;
  p.nvec = (int32_t)(D / 8);
  p.team_threads = pl.team_threads;
  p.teams = pl.teams;
  p.stages = pl.stages;
  p.row_bytes = (uint32_t)(D * xs);
  p.gamma_dtype = a->gamma_dtype;
  p.rout_dtype = a->residual_out_dtype;
  p.nout_dtype = a->norm_out_dtype;
  p.ue8m0 = (a->flags & FARQ_FLAG_UE8M0) ? 1 : 0;
  p.force_timeout = (a->flags & FARQ_FLAG_TEST_FORCE_TIMEOUT) ? 1 : 0;
  p.eps = a->eps;
  p.wait_limit_ns = p.force_timeout ? kTestWaitLimitNs : kWaitLimitNs;

  // Programmatic stream serialisation lets this launch overlap the tail of
  // the previous kernel in the stream; the kernel waits for it
  // (griddepcontrol.wait) before its first global-memory access.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl.grid);
  cfg.blockDim = dim3(pl.team_threads * pl.teams);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, ks.fn, p) != cudaSuccess) return FARQ_ERR_CUDA;
  return FARQ_OK;
}

int farq_ar_launch(const farq_ar_args_t* a, void* stream) {
  if (!a) return FARQ_ERR_NULL_POINTER;
  if (a->struct_size != sizeof(farq_ar_args_t) || a->reserved0 != 0) return FARQ_ERR_BAD_ARGS_SIZE;
  const int64_t M = a->M, D = a->D;
  const int G = a->group_size, W = a->world;
  int st = check_shape(M, D, G);
  if (st != FARQ_OK) return st;
  if (W < 1 || W > kMaxWorld || a->rank < 0 || a->rank >= W) return FARQ_ERR_BAD_SHAPE;
  if (a->x_dtype != FARQ_DTYPE_BF16 && a->x_dtype != FARQ_DTYPE_FP16) return FARQ_ERR_BAD_DTYPE;
  if (!is_float_out(a->gamma_dtype)) return FARQ_ERR_BAD_DTYPE;
  if (a->q_dtype != FARQ_DTYPE_INT8 && a->q_dtype != FARQ_DTYPE_E4M3) return FARQ_ERR_BAD_DTYPE;
  const bool with_norm = a->norm_out[0] != nullptr;
  if (with_norm && !is_float_out(a->norm_out_dtype)) return FARQ_ERR_BAD_DTYPE;
  if (M == 0) return FARQ_OK;
  if (!a->residual || !a->gamma) return FARQ_ERR_NULL_POINTER;
  if (W == 1 && !(a->flags & FARQ_FLAG_AR_KERNEL_AT_WORLD1)) {
    // One rank: the all-reduce is the identity (x = partial[0] exactly), so
    // the single-GPU kernel does the whole call (with its early L2 prefetch
    // and dependent launch); no signal words are used.
    farq_args_t f = {};
    f.struct_size = sizeof(farq_args_t);
    f.x_dtype = a->x_dtype;
    f.gamma_dtype = a->gamma_dtype;
    f.residual_out_dtype = a->x_dtype;
    f.norm_out_dtype = a->norm_out_dtype;
    f.q_dtype = a->q_dtype;
    f.flags = a->flags & (FARQ_FLAG_UE8M0 | FARQ_FLAG_TEST_FORCE_TIMEOUT);
    f.group_size = G;
    f.M = M;
    f.D = D;
    f.eps = a->eps;
    f.x = a->partial[0];
    f.residual = a->residual;
    f.gamma = a->gamma;
    f.residual_out = a->residual_out[0];
    f.norm_out = a->norm_out[0];
    f.x_q = a->x_q[0];
    f.x_scale = a->x_scale[0];
    f.status = a->status;
    return farq_launch(&f, stream);
  }
  if (!aligned(a->residual, 16) || !aligned(a->gamma, 16)) return FARQ_ERR_ALIGNMENT;
  for (int k = 0; k < W; ++k) {
    if (!a->partial[k] || !a->residual_out[k] || !a->x_q[k] || !a->x_scale[k] || !a->signal[k] ||
        (with_norm && !a->norm_out[k]))
      return FARQ_ERR_NULL_POINTER;
    if (!aligned(a->partial[k], 16) || !aligned(a->residual_out[k], 16) || !aligned(a->x_q[k], 8) ||
        !aligned(a->x_scale[k], 4) || !aligned(a->signal[k], 4) ||
        (with_norm && !aligned(a->norm_out[k], 16)))
      return FARQ_ERR_ALIGNMENT;
  }
  int dev, sms, optin;
  if (device_info(&dev, &sms, &optin) != cudaSuccess) return FARQ_ERR_CUDA;
  const int xs = dtype_size(a->x_dtype);
  const uint32_t row_bytes = (uint32_t)(D * xs);
  int K, T;
  st = pick_k(D / 8, 0, false, &K, &T);
  if (st != FARQ_OK) return st;
  const int gl = ilog2(G / 8);
  const bool e4m3 = a->q_dtype == FARQ_DTYPE_E4M3;
  // The kernel compiled for the smallest WMAX in {1, 2, 4, 8} that holds W.
  const int wi = W <= 1 ? 0 : W <= 2 ? 1 : W <= 4 ? 2 : 3;
  using TableFn = ArKernelFn (*)(int, int);
  static const TableFn tables[2][2][4] = {
      {{ar_kernel_bf16_int8_w1, ar_kernel_bf16_int8_w2, ar_kernel_bf16_int8_w4, ar_kernel_bf16_int8_w8},
       {ar_kernel_bf16_e4m3_w1, ar_kernel_bf16_e4m3_w2, ar_kernel_bf16_e4m3_w4, ar_kernel_bf16_e4m3_w8}},
      {{ar_kernel_fp16_int8_w1, ar_kernel_fp16_int8_w2, ar_kernel_fp16_int8_w4, ar_kernel_fp16_int8_w8},
       {ar_kernel_fp16_e4m3_w1, ar_kernel_fp16_e4m3_w2, ar_kernel_fp16_e4m3_w4, ar_kernel_fp16_e4m3_w8}}};
  const int ti = a->x_dtype == FARQ_DTYPE_BF16 ? 0 : 1;
  ArKernelFn fn = tables[ti][e4m3 ? 1 : 0][wi](K, gl);
  const int slot = ((((ti * 2 + (e4m3 ? 1 : 0)) * kMaxK + (K - 1)) * 6 + gl) * 4) + wi;
  int regs = g_ar_regs[dev][slot].load(std::memory_order_relaxed);
  if (regs <= 0) {
    cudaFuncAttributes fa;
    if (cudaFuncGetAttributes(&fa, reinterpret_cast<const void*>(fn)) != cudaSuccess)
      return FARQ_ERR_CUDA;
    regs = fa.numRegs;
    g_ar_regs[dev][slot].store(regs, std::memory_order_relaxed);
  }
  // Row teams as the register file allows (as in the single-GPU kernel); a
  // CTA-wide ring of S >= teams slots of (W + 1) rows, one slot per team.
  const int64_t cap = (int64_t)optin < kSmemPerSm - kSmemReservedPerCta ? optin
                                                                         : kSmemPerSm - kSmemReservedPerCta;
  int teams = kMaxCtaThreads / T;
  const int by_regs = kRegsPerSm / (T * ((regs + 7) / 8 * 8));
  if (by_regs < teams) teams = by_regs;
  if (teams > kMaxTeams) teams = kMaxTeams;
  // The launch shape must be the same on every rank (CTA b meets CTA b), so
  // it is derived from the largest slab, ceil(M / W), not from this rank's.
  const int64_t max_slab = (M + W - 1) / W;
  const int64_t per_sm = (max_slab + sms - 1) / sms;
  if (per_sm < teams) teams = (int)(per_sm < 1 ? 1 : per_sm);
  auto fits = [&](int t, int s) {
    return (int64_t)ar_layout((int)D, row_bytes, W, t, s).total <= cap;
  };
  while (teams > 1 && !fits(teams, teams)) --teams;
  const int S = teams;
  if (teams < 1 || !fits(teams, S)) return FARQ_ERR_UNSUPPORTED;
  int64_t grid = (max_slab + teams - 1) / teams;
  if (grid > sms) grid = sms;
  if (grid > kMaxArCtas) grid = kMaxArCtas;
  if (grid < 1) grid = 1;
  const size_t smem = ar_layout((int)D, row_bytes, W, teams, S).total;
  if ((int)smem > g_ar_smem_set[dev][slot].load(std::memory_order_relaxed)) {
    if (cudaFuncSetAttribute(reinterpret_cast<const void*>(fn),
                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return FARQ_ERR_CUDA;
    g_ar_smem_set[dev][slot].store((int)smem, std::memory_order_relaxed);
  }

  ArParams p = {};
  for (int k = 0; k < W; ++k) {
    p.part[k] = static_cast<const uint8_t*>(a->partial[k]);
    p.rout[k] = static_cast<uint8_t*>(a->residual_out[k]);
    p.nout[k] = with_norm ? static_cast<uint8_t*>(a->norm_out[k]) : nullptr;
    p.q[k] = static_cast<uint8_t*>(a->x_q[k]);
    p.scale[k] = a->x_scale[k];
    p.signal[k] = a->signal[k];
  }
  p.res = static_cast<const uint8_t*>(a->residual);
  p.gamma = a->gamma;
  p.status = a->status;
  // This rank's slab: equal slabs, the M % W remainder one row each to the last ranks.
  const int64_t base = M / W, rem = M % W;
  p.row_begin = a->rank * base + (a->rank > W - rem ? a->rank - (W - rem) : 0);
  p.row_end = p.row_begin + base + (a->rank >= W - rem ? 1 : 0);
  p.D = (int32_t)D;
  p.nvec = (int32_t)(D / 8);
  p.team_threads = T;
  p.teams = teams;
  p.stages = S;
  p.world = W;
  p.rank = a->rank;
  p.row_bytes = row_bytes;
  p.gamma_dtype = a->gamma_dtype;
  p.nout_dtype = a->norm_out_dtype;
  p.ue8m0 = (a->flags & FARQ_FLAG_UE8M0) ? 1 : 0;
  p.epoch = a->epoch;
  p.force_timeout = (a->flags & FARQ_FLAG_TEST_FORCE_TIMEOUT) ? 1 : 0;
  p.eps = a->eps;
  p.wait_limit_ns = p.force_timeout ? kTestWaitLimitNs : kWaitLimitNs;
  void* kargs[] = {&p};
  if (cudaLaunchKernel(reinterpret_cast<const void*>(fn), dim3((unsigned)grid), dim3(T * teams), kargs,
                       smem, static_cast<cudaStream_t>(stream)) != cudaSuccess)
    return FARQ_ERR_CUDA;
  return FARQ_OK;
}

}  // extern "C"
