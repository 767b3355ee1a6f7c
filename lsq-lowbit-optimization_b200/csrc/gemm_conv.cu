// Host side of the tcgen05 W4A8 GEMM and implicit-GEMM convolution:
// argument checks, tile/pipeline sizing, TMA tensor maps, launch.
#include <algorithm>

#include "gemm_w4_kernel.cuh"
#include "gemv_w4.cuh"
#include "launch.cuh"
#include "mma_kernel.cuh"
#include "tensormap.cuh"

namespace w4a8 {

__device__ unsigned g_device_error;

unsigned* device_error_word() {
  static PerDevice<unsigned*> cached;
  int dev = 0;
  cudaGetDevice(&dev);
  if (unsigned* c = cached.get(dev)) return c;
  void* ptr = nullptr;
  if (cudaGetSymbolAddress(&ptr, g_device_error) != cudaSuccess) return nullptr;
  cached.set(dev, static_cast<unsigned*>(ptr));
  return static_cast<unsigned*>(ptr);
}

namespace {

constexpr int kSmemAttr = 226 * 1024;         // dynamic smem requested per CTA
constexpr int kSmemBudget = kSmemAttr - 1024;  // minus base-alignment slack

template <int BN, bool I4, bool CV, bool PL = false>
int launch_t(const CUtensorMap& tA, const CUtensorMap& tW, const CUtensorMap* tH, const KParams& p, int grid,
             cudaStream_t st) {
  auto kern = w4a8_mma_kernel<BN, I4, CV, PL>;
  static PerDevice<bool> attr_done;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_done.get(dev)) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemAttr) != cudaSuccess)
      return W4A8_ERR_LAUNCH;
    attr_done.set(dev, true);
  }
  if (launch_kernel(kern, dim3(unsigned(grid)), dim3(Roles<CV>::kThreads), kSmemAttr, st, tA, tW, tH[0], tH[1], tH[2],
                    tH[3], p) != cudaSuccess)
    return W4A8_ERR_LAUNCH;
  return cudaGetLastError() == cudaSuccess ? W4A8_OK : W4A8_ERR_LAUNCH;
}

template <int BN, int CTA, bool SWAP>
int launch_w4_t(const CUtensorMap& tA, const CUtensorMap& tW, const KParams& p, int grid, cudaStream_t st) {
  auto kern = w4a8_gemm_w4_kernel<BN, CTA, SWAP>;
  static PerDevice<bool> attr_done;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_done.get(dev)) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemAttr) != cudaSuccess)
      return W4A8_ERR_LAUNCH;
    attr_done.set(dev, true);
  }
  cudaLaunchConfig_t cfg;
  std::memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3(unsigned(grid > 0 ? grid : 2 * 148), 1, 1);
  cfg.blockDim = dim3(kW4Threads, 1, 1);
  cfg.dynamicSmemBytes = kSmemAttr;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = CTA;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (grid < 0) {  // query: co-resident clusters
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) != cudaSuccess) return 0;
    return clusters;
  }
  if (launch_kernel_attrs(kern, cfg.gridDim, cfg.blockDim, kSmemAttr, st, attr, 1, tA, tW, p) != cudaSuccess)
    return W4A8_ERR_LAUNCH;
  return cudaGetLastError() == cudaSuccess ? W4A8_OK : W4A8_ERR_LAUNCH;
}

int launch_w4(int bn, int cta, bool swap, const CUtensorMap& tA, const CUtensorMap& tW, const KParams& p, int grid,
              cudaStream_t st) {
  if (cta == 2) return launch_w4_t<256, 2, false>(tA, tW, p, grid, st);
  if (swap) {
    switch (bn) {
      case 32: return launch_w4_t<32, 1, true>(tA, tW, p, grid, st);
      case 64: return launch_w4_t<64, 1, true>(tA, tW, p, grid, st);
      case 128: return launch_w4_t<128, 1, true>(tA, tW, p, grid, st);
      default: return W4A8_ERR_UNSUPPORTED;
    }
  }
  switch (bn) {
    case 64: return launch_w4_t<64, 1, false>(tA, tW, p, grid, st);
    case 128: return launch_w4_t<128, 1, false>(tA, tW, p, grid, st);
    case 256: return launch_w4_t<256, 1, false>(tA, tW, p, grid, st);
    default: return W4A8_ERR_UNSUPPORTED;
  }
}

// Co-resident CTA pairs of the pair W4 GEMM on the current device (cached).
int pair_slots() {
  static PerDevice<int> cached;
  int dev = 0;
  cudaGetDevice(&dev);
  if (const int c = cached.get(dev)) return c;
  CUtensorMap dummy;
  std::memset(&dummy, 0, sizeof(dummy));
  KParams p;
  std::memset(&p, 0, sizeof(p));
  const int n = launch_w4(256, 2, false, dummy, dummy, p, -1, nullptr);
  if (n > 0) cached.set(dev, n);
  return n > 0 ? n : 0;
}

template <bool I4, bool CV>
int launch_bn(int bn, const CUtensorMap& tA, const CUtensorMap& tW, const CUtensorMap* tH, const KParams& p,
              int grid, cudaStream_t st) {
  switch (bn) {
    case 64: return launch_t<64, I4, CV>(tA, tW, tH, p, grid, st);
    case 128: return launch_t<128, I4, CV>(tA, tW, tH, p, grid, st);
    case 256: return launch_t<256, I4, CV>(tA, tW, tH, p, grid, st);
    default: return W4A8_ERR_UNSUPPORTED;
  }
}

int launch(bool i4, bool cv, int bn, const CUtensorMap& tA, const CUtensorMap& tW, const CUtensorMap* tH,
           const KParams& p, int grid, cudaStream_t st) {
  if (i4) return cv ? launch_bn<true, true>(bn, tA, tW, tH, p, grid, st)
                    : launch_bn<true, false>(bn, tA, tW, tH, p, grid, st);
  return cv ? launch_bn<false, true>(bn, tA, tW, tH, p, grid, st)
            : launch_bn<false, false>(bn, tA, tW, tH, p, grid, st);
}

int check_epilogue(const w4a8_epilogue* e) {
  if (!e) return W4A8_ERR_ARG;
  if (e->out_kind < W4A8_OUT_S32 || e->out_kind > W4A8_OUT_S8) return W4A8_ERR_ARG;
  if (e->out_kind == W4A8_OUT_S8) {
    if (!(e->out_scale > 0.0f)) return W4A8_ERR_ARG;
    if (e->qn < -128 || e->qp > 127 || e->qn > e->qp) return W4A8_ERR_ARG;
  }
  return W4A8_OK;
}

void fill_epi(EpiParams& d, const w4a8_epilogue* e, void* out, int n_total) {
  d.out = out;
  d.out_kind = e->out_kind;
  d.relu = e->relu;
  d.alpha = e->alpha;
  d.alpha_scalar = e->alpha_scalar;
  d.beta = e->beta;
  d.residual = e->residual;
  d.res_ld = e->res_ld;
  d.out_scale = e->out_scale;
  d.qn = e->qn;
  d.qp = e->qp;
  d.aux = e->aux;
  d.aux_ld = e->aux_ld;
  d.n_total = n_total;
  d.vec16 = 0;
  d.v8 = 0;
}

// Sets vec16 once the output strides are known: the epilogue may then skip
// its per-chunk shape and alignment checks.
void set_vec16(EpiParams& d) {
  auto al = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  const long long esz = d.out_kind == 1 ? 4 : (d.out_kind == 2 ? 2 : 1);
  d.vec16 = d.out_kind != 0 && d.s_ch == 1 && d.n_total % 16 == 0 && al(d.out) && (d.s_pix * esz) % 16 == 0 &&
            (d.s_img * esz) % 16 == 0 && (!d.alpha || al(d.alpha)) && (!d.beta || al(d.beta)) &&
            (!d.residual || (al(d.residual) && d.res_ld % 4 == 0)) && (!d.aux || (al(d.aux) && d.aux_ld % 4 == 0));
  // 256-bit float32 accesses: 32-byte aligned bases and strides of 8 floats.
  auto al32 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 31) == 0; };
  d.v8 = d.vec16 && (!d.residual || (al32(d.residual) && d.res_ld % 8 == 0)) &&
         (!d.aux || (al32(d.aux) && d.aux_ld % 8 == 0)) &&
         (d.out_kind != 1 || (al32(d.out) && d.s_pix % 8 == 0 && d.s_img % 8 == 0));
}

int pick_stages(uint32_t per_stage, uint32_t reserved) {
  if (reserved + 2 * per_stage > static_cast<uint32_t>(kSmemBudget)) return 0;
  return std::min<int>(kMaxStages, (kSmemBudget - reserved) / per_stage);
}

int floordiv(int a, int b) { return a >= 0 ? a / b : -((-a + b - 1) / b); }

// A few tokens (M <= 8, K a multiple of 64, activations fit in shared
// memory) run on the CUDA-core GEMV, which streams the packed weights
// straight into registers.
bool use_gemv(int M, int K) {
  return M >= 1 && M <= kGemvMaxTokens && K % 64 == 0 && gemv_smem_bytes(kGemvMaxTokens, K) <= 200 * 1024;
}

template <int MT, bool ROWS>
int launch_gemv_t(const int8_t* A, int64_t lda, const void* W, int64_t ldw, int M, int N, int K,
                  const EpiParams& e, cudaStream_t st) {
  auto kern = ROWS ? w4a8_gemv_w4_rows_kernel<MT> : w4a8_gemv_w4_kernel<MT>;
  const size_t smem = ROWS ? gemv_rows_smem_bytes(MT, K) : gemv_smem_bytes(MT, K);
  if (smem > 48 * 1024 && cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != cudaSuccess)
    return W4A8_ERR_LAUNCH;
  const int per_block = ROWS ? kGemvRows : 32;
  const dim3 grid(unsigned((N + per_block - 1) / per_block), ROWS ? 1u : unsigned((M + MT - 1) / MT));
  if (launch_kernel(kern, grid, dim3(kGemvWarps * 32), smem, st, A, lda, static_cast<const uint8_t*>(W), ldw, M, N,
                    K, e) != cudaSuccess)
    return W4A8_ERR_LAUNCH;
  return cudaGetLastError() == cudaSuccess ? W4A8_OK : W4A8_ERR_LAUNCH;
}

#ifndef W4A8_GEMV_TOKENS_MACS
#define W4A8_GEMV_TOKENS_MACS 1.5e8
#endif
// Small GEMMs with 9..128 tokens whose tensor-core tiles could not fill
// half the GPU and whose multiply-adds take the CUDA cores a few
// microseconds: 8-token groups of the lane-per-row GEMV. The tensor-core
// path is latency-bound there (TMEM allocation, pipeline ramp and epilogue
// of a handful of k-blocks per CTA). Measured in CUDA graphs, weights in L2:
// 16x2048x2048 10.6 -> 7.7 us, 32x1024x1024 8.9 -> 6.5, 64x1024x2048
// 12.2 -> 10.4, 128x512x512 7.8 -> 6.7; at 256 tokens (256x1000x512) the
// token groups cost more than they save (9.8 -> 23.8 us), hence the limit.
bool use_gemv_tokens(int M, int N, int K, int sms) {
  if (M <= kGemvMaxTokens || M > 128 || K % 64 || gemv_smem_bytes(kGemvMaxTokens, K) > 200 * 1024) return false;
  const long long tiles = (long long)((M + kBM - 1) / kBM) * ((N + 63) / 64);
  return tiles < sms / 2 && double(M) * double(N) * double(K) <= W4A8_GEMV_TOKENS_MACS;
}

int gemv_w4(const int8_t* A, int64_t lda, const void* W, int64_t ldw, int M, int N, int K,
            const w4a8_epilogue* epi, void* C, int64_t ldc, cudaStream_t st) {
  EpiParams e;
  std::memset(&e, 0, sizeof(e));
  fill_epi(e, epi, C, N);
  e.acc_fits_22 = (double)K * 128.0 * 8.0 < 4194304.0;
  e.s_img = 0;
  e.s_pix = ldc;
  e.s_ch = 1;
  if (M <= 1) return launch_gemv_t<1, true>(A, lda, W, ldw, M, N, K, e, st);
  if (M <= 2) return launch_gemv_t<2, true>(A, lda, W, ldw, M, N, K, e, st);
  if (M <= 4) return launch_gemv_t<4, false>(A, lda, W, ldw, M, N, K, e, st);
  return launch_gemv_t<8, false>(A, lda, W, ldw, M, N, K, e, st);
}

// Split-K plan for a small-M (<= 128) W4 GEMM whose output tiles alone
// cannot fill the GPU. Tiles are 128 channels x bn tokens (bn = 32, 64 or
// 128 covering M, swapped operands); about four work units per SM, each at
// least two k-blocks long. Returns the number of splits (0: no split).
int splitk_plan(int M, int N, int K, int sms, int& bn, int& kb_per) {
  const int num_kb = (K + kBK - 1) / kBK;
  if (M > 64 || num_kb < 16 || use_gemv(M, K)) return 0;
  bn = M <= 32 ? 32 : (M <= 64 ? 64 : 128);
  const int tiles = (N + kBM - 1) / kBM;
  if (tiles >= sms || num_kb < 4) return 0;
  int s = std::max(1, std::min(4 * sms / tiles, num_kb / 2));
  kb_per = (num_kb + s - 1) / s;
  s = (num_kb + kb_per - 1) / kb_per;
  return s > 1 ? s : 0;
}

// W4 GEMM on the three-ring kernel; CTA pairs (256 x 256 tiles) when there
// are enough of them to fill the GPU; split-K into `ws` (int32 [M, N],
// ws_bytes) when a workspace is given and the tiles are too few.
int gemm_w4(const int8_t* A, int64_t lda, const void* W, int64_t ldw, int M, int N, int K,
            const w4a8_epilogue* epi, void* C, int64_t ldc, int bn, int sms, int* ws, size_t ws_bytes,
            cudaStream_t stream) {
  if (use_gemv(M, K) || use_gemv_tokens(M, N, K, sms)) return gemv_w4(A, lda, W, ldw, M, N, K, epi, C, ldc, stream);
  int kb_per = 0, bn_split = bn;
  const int splits = ws ? splitk_plan(M, N, K, sms, bn_split, kb_per) : 0;
  if (splits && ws_bytes < size_t(M) * size_t(N) * 4) return W4A8_ERR_ARG;
  const int pair_tiles = ((M + 2 * kBM - 1) / (2 * kBM)) * ((N + 255) / 256);
  const int slots = (!splits && N >= 256 && M > kBM && pair_tiles >= sms / 2) ? pair_slots() : 0;
  const int cta = slots > 0 ? 2 : 1;
  if (cta == 2) bn = 256;
  const bool swap = splits > 0;  // split-K runs with swapped operands (see splitk_plan)
  if (swap) bn = bn_split;
  const int bnl = swap ? kBM : bn / cta;  // weight rows per CTA
  const int xrows = swap ? bn : kBM;      // activation rows per stage

  KParams p;
  std::memset(&p, 0, sizeof(p));
  p.M = M;
  p.N = N;
  p.num_kb = (K + kBK - 1) / kBK;
  p.tiles_m = swap ? (M + bn - 1) / bn : (cta == 2 ? (M + 2 * kBM - 1) / (2 * kBM) : (M + kBM - 1) / kBM);
  p.tiles_n = swap ? (N + kBM - 1) / kBM : (N + bn - 1) / bn;
  p.k_splits = splits ? splits : 1;
  p.kb_per_split = splits ? kb_per : p.num_kb;
  p.ws = splits ? ws : nullptr;
  p.ws_ld = N;
  // Ring depths: four packed stages (weight bytes arrive far ahead of use),
  // then A and int8 B stages added in step (A first) while they fit; the
  // int8 ring covers MMA completion -> unpack -> proxy fence -> arrive.
  const int64_t a_bytes = int64_t(xrows) * kBK, pk_bytes = int64_t(bnl) * (kBK / 2), b8_bytes = int64_t(bnl) * kBK;
  int sa = 2, sp = 4, sb = 2;
  int64_t left = kSmemBudget - sa * a_bytes - sp * pk_bytes - sb * b8_bytes;
  if (left < 0) return W4A8_ERR_UNSUPPORTED;
  for (bool grew = true; grew;) {
    grew = false;
    if (sa < kMaxStages && left >= a_bytes) { ++sa; left -= a_bytes; grew = true; }
    if (sb < kMaxB8Stages && left >= b8_bytes) { ++sb; left -= b8_bytes; grew = true; }
  }
  while (sp < kMaxPkStages && left >= pk_bytes) { ++sp; left -= pk_bytes; }
  p.stages = sa;
  p.pk_stages = sp;
  p.b8_stages = sb;
  p.a_off = 0;
  p.a_stage_bytes = uint32_t(a_bytes);
  p.bp_off = uint32_t(sa * a_bytes);
  p.bp_stage_bytes = uint32_t(pk_bytes);
  p.b_off = uint32_t(p.bp_off + sp * pk_bytes);  // a multiple of 1024 (128-byte swizzle atoms)
  p.b_stage_bytes = uint32_t(b8_bytes);
  p.err = device_error_word();
  if (!p.err) return W4A8_ERR_LAUNCH;
  fill_epi(p.epi, epi, C, N);
  p.epi.acc_fits_22 = (double)K * 128.0 * 8.0 < 4194304.0;  // |acc| <= K * 128 * 8
  p.epi.s_img = 0;
  p.epi.s_pix = ldc;
  p.epi.s_ch = 1;
  set_vec16(p.epi);

  CUtensorMap tA, tW;
  {
    const uint64_t dims[2] = {uint64_t(K), uint64_t(M)};
    const uint64_t str[1] = {uint64_t(lda)};
    const uint32_t box[2] = {uint32_t(kBK), uint32_t(xrows)};
    if (encode_u8(&tA, A, 2, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B)) return W4A8_ERR_TENSORMAP;
  }
  {
    const uint64_t dims[2] = {uint64_t(K / 2), uint64_t(N)};
    const uint64_t str[1] = {uint64_t(ldw)};
    const uint32_t box[2] = {uint32_t(kBK / 2), uint32_t(bnl)};
    if (encode_u8(&tW, W, 2, dims, str, box, CU_TENSOR_MAP_SWIZZLE_NONE)) return W4A8_ERR_TENSORMAP;
  }
  const int units = p.tiles_m * p.tiles_n * p.k_splits;
  const int grid = cta == 2 ? 2 * std::min(units, slots) : std::min(units, sms);
  if (splits && cudaMemsetAsync(ws, 0, size_t(M) * size_t(N) * 4, stream) != cudaSuccess) return W4A8_ERR_LAUNCH;
  if (int rc = launch_w4(bn, cta, swap, tA, tW, p, grid, stream)) return rc;
  if (!splits) return W4A8_OK;
  const long long threads = (long long)M * ((N + 15) / 16);
  if (launch_kernel(w4a8_splitk_finish_kernel, dim3(unsigned((threads + 255) / 256)), dim3(256), 0, stream, p) !=
      cudaSuccess)
    return W4A8_ERR_LAUNCH;
  return cudaGetLastError() == cudaSuccess ? W4A8_OK : W4A8_ERR_LAUNCH;
}

}  // namespace
}  // namespace w4a8

using namespace w4a8;

extern "C" int w4a8_abi_version(void) { return W4A8_ABI_VERSION; }
extern "C" int w4a8_num_sms(void) { return device_sms(); }

extern "C" int w4a8_device_error(unsigned* bits) {
  if (cudaDeviceSynchronize() != cudaSuccess) return W4A8_ERR_LAUNCH;
  unsigned* word = device_error_word();
  if (!word) return W4A8_ERR_LAUNCH;
  unsigned v = 0;
  if (cudaMemcpy(&v, word, sizeof(v), cudaMemcpyDeviceToHost) != cudaSuccess) return W4A8_ERR_LAUNCH;
  if (bits) *bits = v;
  if (v) {
    const unsigned zero = 0;
    cudaMemcpy(word, &zero, sizeof(zero), cudaMemcpyHostToDevice);
    return W4A8_ERR_DEVICE;
  }
  return W4A8_OK;
}

namespace {
// Shared argument checks of the GEMM entry points; W4A8_OK + *empty when
// there is nothing to compute.
int check_gemm(const int8_t* A, int64_t lda, const void* W, int64_t ldw, int w_kind, int M, int N, int K,
               const w4a8_epilogue* epi, const void* C, int64_t ldc, bool* empty) {
  *empty = false;
  if (M < 0 || N < 0 || K <= 0) return W4A8_ERR_ARG;
  if (w_kind != W4A8_W_INT8 && w_kind != W4A8_W_INT4) return W4A8_ERR_ARG;
  const bool i4 = w_kind == W4A8_W_INT4;
  if (i4 && (K & 1)) return W4A8_ERR_ARG;
  if (int rc = check_epilogue(epi)) return rc;
  if (M == 0 || N == 0) {
    *empty = true;
    return W4A8_OK;
  }
  if (!A || !W || !C) return W4A8_ERR_ARG;
  if (lda < K || ldw < (i4 ? K / 2 : K) || ldc < N) return W4A8_ERR_ARG;
  if ((lda % 16) || (ldw % 16) || !aligned16(A) || !aligned16(W)) return W4A8_ERR_ALIGN;
  return W4A8_OK;
}
}  // namespace

extern "C" int w4a8_gemm_splitk_workspace(int M, int N, int K, int w_kind, size_t* bytes) {
  if (!bytes || M < 0 || N < 0 || K <= 0) return W4A8_ERR_ARG;
  int bn = 0, kb_per = 0;
  const bool split = w_kind == W4A8_W_INT4 && M > 0 && N > 0 && splitk_plan(M, N, K, device_sms(), bn, kb_per) > 0;
  *bytes = split ? size_t(M) * size_t(N) * 4 : 0;
  return W4A8_OK;
}

extern "C" int w4a8_gemm_splitk(const int8_t* A, int64_t lda, const void* W, int64_t ldw, int w_kind, int M, int N,
                                int K, const w4a8_epilogue* epi, void* C, int64_t ldc, void* workspace,
                                size_t workspace_bytes, void* stream) {
  bool empty = false;
  if (int rc = check_gemm(A, lda, W, ldw, w_kind, M, N, K, epi, C, ldc, &empty)) return rc;
  if (empty) return W4A8_OK;
  if (w_kind != W4A8_W_INT4 || !workspace) return w4a8_gemm(A, lda, W, ldw, w_kind, M, N, K, epi, C, ldc, stream);
  if (!aligned16(workspace)) return W4A8_ERR_ALIGN;
  const int sms = device_sms();
  const int tiles_m = (M + kBM - 1) / kBM;
  int bn = N > 128 ? 256 : (N > 64 ? 128 : 64);
  while (bn > 64 && tiles_m * ((N + bn - 1) / bn) < sms) bn >>= 1;
  return gemm_w4(A, lda, W, ldw, M, N, K, epi, C, ldc, bn, sms, static_cast<int*>(workspace), workspace_bytes,
                 static_cast<cudaStream_t>(stream));
}

namespace {
// Scratch of w4a8_gemm_splitk_noalloc, for callers that cannot allocate
// device memory: the split-K int32 partial sums live in this fixed array
// instead of a workspace. Every GPU that loads the library holds it until the
// process exits. In host code the name is only a stand-in for the symbol, not
// a device address: kernels get the address from noalloc_scratch().
static __device__ __align__(256) int g_splitk_scratch[W4A8_NOALLOC_SCRATCH_BYTES / 4];

// Device address of g_splitk_scratch on the current device, looked up on the
// first call per device (cudaGetSymbolAddress, return code checked) and cached.
int* noalloc_scratch() {
  static PerDevice<int*> cached;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  if (int* c = cached.get(dev)) return c;
  void* ptr = nullptr;
  if (cudaGetSymbolAddress(&ptr, g_splitk_scratch) != cudaSuccess) return nullptr;
  cached.set(dev, static_cast<int*>(ptr));
  return static_cast<int*>(ptr);
}
}  // namespace

extern "C" int w4a8_gemm_splitk_noalloc(const int8_t* A, int64_t lda, const void* W, int64_t ldw, int w_kind,
                                        int M, int N, int K, const w4a8_epilogue* epi, void* C, int64_t ldc,
                                        void* stream) {
  bool empty = false;
  if (int rc = check_gemm(A, lda, W, ldw, w_kind, M, N, K, epi, C, ldc, &empty)) return rc;
  if (empty) return W4A8_OK;
  if (w_kind != W4A8_W_INT4) return W4A8_ERR_ARG;
  const int sms = device_sms();
  const int tiles_m = (M + kBM - 1) / kBM;
  int bn = N > 128 ? 256 : (N > 64 ? 128 : 64);
  while (bn > 64 && tiles_m * ((N + bn - 1) / bn) < sms) bn >>= 1;
  // Only a split-K shape touches the scratch array; the others (few-token
  // GEMV, or enough output tiles to fill the GPU) run unsplit, as w4a8_gemm.
  int split_bn = 0, kb_per = 0;
  if (splitk_plan(M, N, K, sms, split_bn, kb_per) == 0)
    return gemm_w4(A, lda, W, ldw, M, N, K, epi, C, ldc, bn, sms, nullptr, 0, static_cast<cudaStream_t>(stream));
  if (int64_t(M) * int64_t(N) * 4 > int64_t(W4A8_NOALLOC_SCRATCH_BYTES)) return W4A8_ERR_ARG;
  int* scratch = noalloc_scratch();
  if (!scratch) return W4A8_ERR_LAUNCH;
  // gemm_w4 zeroes the M x N sums it uses (cudaMemsetAsync) before the kernel.
  return gemm_w4(A, lda, W, ldw, M, N, K, epi, C, ldc, bn, sms, scratch, W4A8_NOALLOC_SCRATCH_BYTES,
                 static_cast<cudaStream_t>(stream));
}

extern "C" int w4a8_gemm(const int8_t* A, int64_t lda, const void* W, int64_t ldw, int w_kind, int M, int N,
                         int K, const w4a8_epilogue* epi, void* C, int64_t ldc, void* stream) {
  bool empty = false;
  if (int rc = check_gemm(A, lda, W, ldw, w_kind, M, N, K, epi, C, ldc, &empty)) return rc;
  if (empty) return W4A8_OK;
  const bool i4 = w_kind == W4A8_W_INT4;

  const int sms = device_sms();
  const int tiles_m = (M + kBM - 1) / kBM;
  int bn = N > 128 ? 256 : (N > 64 ? 128 : 64);
  while (bn > 64 && tiles_m * ((N + bn - 1) / bn) < sms) bn >>= 1;
  if (i4) return gemm_w4(A, lda, W, ldw, M, N, K, epi, C, ldc, bn, sms, nullptr, 0, static_cast<cudaStream_t>(stream));

  KParams p;
  std::memset(&p, 0, sizeof(p));
  p.M = M;
  p.N = N;
  p.num_kb = (K + kBK - 1) / kBK;
  p.tiles_m = tiles_m;
  p.tiles_n = (N + bn - 1) / bn;
  // Packed int4 weights land in the upper half of the int8 B stage and are
  // expanded in place, so a stage is A (16 KB) + B (bn x 128 B).
  p.a_stage_bytes = kBM * kBK;
  p.b_stage_bytes = bn * kBK;
  p.bp_stage_bytes = 0;
  const uint32_t per_stage = p.a_stage_bytes + p.b_stage_bytes;
  p.stages = pick_stages(per_stage, 0);
  if (p.stages < 2) return W4A8_ERR_UNSUPPORTED;
  p.halo_stages = 0;
  p.a_off = 0;
  p.b_off = p.a_off + p.stages * p.a_stage_bytes;
  p.bp_off = 0;
  p.h_off = p.b_off + p.stages * p.b_stage_bytes;
  p.tx_bytes = p.a_stage_bytes + (i4 ? p.b_stage_bytes / 2 : p.b_stage_bytes);
  p.tmem_cols = 2 * bn < 32 ? 32 : 2 * bn;
  p.err = device_error_word();
  if (!p.err) return W4A8_ERR_LAUNCH;
  fill_epi(p.epi, epi, C, N);
  // |acc| <= K * 128 * max|w|; below 2^22 the epilogue skips its range check.
  p.epi.acc_fits_22 = (double)K * 128.0 * (i4 ? 8.0 : 128.0) < 4194304.0;
  p.epi.s_img = 0;
  p.epi.s_pix = ldc;
  p.epi.s_ch = 1;
  set_vec16(p.epi);

  CUtensorMap tA, tW, tH[4];
  std::memset(tH, 0, sizeof(tH));
  {
    const uint64_t dims[2] = {uint64_t(K), uint64_t(M)};
    const uint64_t str[1] = {uint64_t(lda)};
    const uint32_t box[2] = {uint32_t(kBK), uint32_t(kBM)};
    if (encode_u8(&tA, A, 2, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B)) return W4A8_ERR_TENSORMAP;
  }
  {
    const uint64_t dims[2] = {uint64_t(i4 ? K / 2 : K), uint64_t(N)};
    const uint64_t str[1] = {uint64_t(ldw)};
    const uint32_t box[2] = {uint32_t(i4 ? kBK / 2 : kBK), uint32_t(bn)};
    if (encode_u8(&tW, W, 2, dims, str, box, i4 ? CU_TENSOR_MAP_SWIZZLE_NONE : CU_TENSOR_MAP_SWIZZLE_128B))
      return W4A8_ERR_TENSORMAP;
  }
  const int grid = std::min(p.tiles_m * p.tiles_n, sms);
  return launch(i4, false, bn, tA, tW, tH, p, grid, static_cast<cudaStream_t>(stream));
}

extern "C" int w4a8_conv2d(const int8_t* x, const void* W, int w_kind, int64_t ldw, const w4a8_conv_geom* g,
                           const w4a8_epilogue* epi, void* out, void* stream) {
  if (!g) return W4A8_ERR_ARG;
  if (w_kind != W4A8_W_INT8 && w_kind != W4A8_W_INT4) return W4A8_ERR_ARG;
  const bool i4 = w_kind == W4A8_W_INT4;
  if (int rc = check_epilogue(epi)) return rc;
  if (g->n < 0 || g->h < 1 || g->w < 1 || g->c < 16 || g->kh < 1 || g->kw < 1 || g->ho < 1 || g->wo < 1 ||
      g->o < 1 || g->pad_h < 0 || g->pad_w < 0)
    return W4A8_ERR_ARG;
  if (g->stride != 1 && g->stride != 2) return W4A8_ERR_UNSUPPORTED;
  if (g->c % 16) return W4A8_ERR_ALIGN;
  // Halo pixels are 16/32/64/128-byte rows (swizzle widths); wider inputs
  // are split into groups of 128 channels.
  if (g->c != 16 && g->c != 32 && g->c != 64 && g->c % 128) return W4A8_ERR_UNSUPPORTED;
  if (g->out_layout != W4A8_LAYOUT_NHWC && g->out_layout != W4A8_LAYOUT_NCHW) return W4A8_ERR_ARG;
  if (g->out_layout == W4A8_LAYOUT_NHWC && g->ldo < g->o) return W4A8_ERR_ARG;
  if (g->pool != 0 && g->pool != 1) return W4A8_ERR_ARG;
  if (g->pool && (i4 || g->o > 64 || g->out_layout != W4A8_LAYOUT_NHWC || epi->residual ||
                  (epi->out_kind != W4A8_OUT_S8 && epi->out_kind != W4A8_OUT_F32) || (g->o % 4)))
    return W4A8_ERR_UNSUPPORTED;
  // The pooled epilogue reads alpha / beta and stores in 4-channel vectors.
  if (g->pool && ((reinterpret_cast<uintptr_t>(out) & (epi->out_kind == W4A8_OUT_F32 ? 15 : 3)) || (g->ldo % 4) ||
                  (epi->aux && ((reinterpret_cast<uintptr_t>(epi->aux) & 15) || (epi->aux_ld % 4))) ||
                  (reinterpret_cast<uintptr_t>(epi->alpha) & 15) || (reinterpret_cast<uintptr_t>(epi->beta) & 15)))
    return W4A8_ERR_ALIGN;
  if (g->n == 0) return W4A8_OK;
  if (!x || !W || !out) return W4A8_ERR_ARG;
  const int s = g->stride;
  const int taps = g->kh * g->kw;
  const long long k_total = (long long)taps * g->c;
  if (ldw < (i4 ? k_total / 2 : k_total)) return W4A8_ERR_ARG;
  if ((ldw % 16) || !aligned16(x) || !aligned16(W)) return W4A8_ERR_ALIGN;
  // Every output pixel must read at least one in-bounds row/column window.
  if ((long long)(g->ho - 1) * s - g->pad_h >= g->h || (long long)(g->wo - 1) * s - g->pad_w >= g->w)
    return W4A8_ERR_ARG;

  // Halo pixels are stored channel-group-major like NHWC: one pixel = cg
  // bytes, 128/64/32-byte rows swizzled to match (16-byte rows unswizzled).
  const int cg = g->c < 128 ? g->c : 128;
  const int groups = g->c / cg;
  const int kbpg = (taps * cg + kBK - 1) / kBK;
  const int steps = kbpg * (kBK / 32);
  if (steps > kMaxSteps) return W4A8_ERR_UNSUPPORTED;

  // Stride phases (sub-tiles) and their offsets in phase-view units.
  int qmin_h[2] = {1 << 20, 1 << 20}, qmax_h[2] = {-(1 << 20), -(1 << 20)};
  int qmin_w[2] = {1 << 20, 1 << 20}, qmax_w[2] = {-(1 << 20), -(1 << 20)};
  bool used[2][2] = {{false, false}, {false, false}};
  for (int ky = 0; ky < g->kh; ++ky)
    for (int kx = 0; kx < g->kw; ++kx) {
      const int dy = ky - g->pad_h, dx = kx - g->pad_w;
      const int qy = floordiv(dy, s), py = dy - qy * s;
      const int qx = floordiv(dx, s), px = dx - qx * s;
      used[py][px] = true;
      qmin_h[py] = std::min(qmin_h[py], qy);
      qmax_h[py] = std::max(qmax_h[py], qy);
      qmin_w[px] = std::min(qmin_w[px], qx);
      qmax_w[px] = std::max(qmax_w[px], qx);
    }
  int span_h = 0, span_w = 0;
  for (int i = 0; i < s; ++i) {
    if (qmax_h[i] >= qmin_h[i]) span_h = std::max(span_h, qmax_h[i] - qmin_h[i]);
    if (qmax_w[i] >= qmin_w[i]) span_w = std::max(span_w, qmax_w[i] - qmin_w[i]);
  }
  KParams p;
  std::memset(&p, 0, sizeof(p));
  ConvParams& cp = p.conv;
  cp.ho = g->ho;
  cp.wo = g->wo;
  cp.pool = g->pool;
  if (g->pool) {
    cp.pho = (g->ho - 1) / 2 + 1;
    cp.pwo = (g->wo - 1) / 2 + 1;
    cp.tiles_h = (cp.pho + kPoolRows - 1) / kPoolRows;
    cp.tiles_w = (cp.pwo + kPoolCols - 1) / kPoolCols;
  } else {
    cp.tiles_h = (g->ho + kTileH - 1) / kTileH;
    cp.tiles_w = (g->wo + kTileW - 1) / kTileW;
  }
  // Outputs of at most 8x8 (ResNet's 7x7 stage) fill a 16x8 tile to 38%:
  // such tiles hold two images instead (each an 8x8 block; with stride 2
  // every phase view is packed the same way).
  cp.n = g->n;
  cp.pack2 = (!g->pool && g->ho <= 8 && g->wo <= kTileW) ? 1 : 0;
  const int sub_h = cp.pack2 ? kTileH / 2 : kTileH;  // output rows per image in a tile
  if (cp.pack2) cp.tiles_h = cp.tiles_w = 1;
  const int img_mult = cp.pack2 ? 2 : 1;              // images interleaved in a halo row
  cp.cg = cg;
  cp.a_layout = cg == 128 ? kLayoutSw128 : cg == 64 ? kLayoutSw64 : cg == 32 ? kLayoutSw32 : kLayoutNone;
  cp.halo_w = kTileW + span_w;
  cp.halo_h = sub_h + span_h;
  // One TMA request per halo row instead of one per 16-byte pixel.
  cp.wc_bytes = (g->c == 16 && s == 1 && !cp.pack2 && cp.halo_w * 16 <= 256) ? 16 : 0;
  if (cp.halo_w > 256 || cp.halo_h > 256) return W4A8_ERR_UNSUPPORTED;
  cp.slot_bytes = (uint32_t(img_mult * cp.halo_w * cp.halo_h * cg) + 1023u) & ~1023u;
  int slot_of[2][2] = {{-1, -1}, {-1, -1}};
  int slot_py[4], slot_px[4];
  int ns = 0;
  for (int py = 0; py < s; ++py)
    for (int px = 0; px < s; ++px)
      if (used[py][px]) {
        slot_of[py][px] = ns;
        slot_py[ns] = py;
        slot_px[ns] = px;
        cp.slot_qh[ns] = qmin_h[py];
        cp.slot_qw[ns] = qmin_w[px];
        ++ns;
      }
  cp.n_slots = ns;
  cp.halo_bytes = (cp.slot_bytes * ns + 1023u) & ~1023u;
  // The pooled conv loads a tile pair into each halo stage.
  cp.tile_halo_bytes = cp.halo_bytes;
  if (g->pool) cp.halo_bytes *= 2;
  cp.halo_tx_bytes = uint32_t(ns * img_mult * cp.halo_w * cp.halo_h * cg);
  cp.kb_per_group = kbpg;
  cp.tail_steps = (taps * cg + 31) / 32 - (kbpg - 1) * (kBK / 32);
  auto chunk_off = [&](int k) -> long long {
    const int t = k / cg, within = k % cg;
    const int ky = t / g->kw, kx = t % g->kw;
    const int dy = ky - g->pad_h, dx = kx - g->pad_w;
    const int qy = floordiv(dy, s), py = dy - qy * s;
    const int qx = floordiv(dx, s), px = dx - qx * s;
    const int sl = slot_of[py][px];
    const int pix = (qy - qmin_h[py]) * img_mult * cp.halo_w + (qx - qmin_w[px]);
    return (long long)sl * cp.slot_bytes + (long long)pix * cg + within;
  };
  // One operand descriptor per 32-byte K-step, relative to the halo stage
  // base; steps past the real K repeat step 0 (their weights are zero).
  const uint32_t sbo = uint32_t(cp.halo_w * cg);
  for (int j = 0; j < steps; ++j) {
    const int k = 32 * j;
    if (k >= taps * cg) {
      cp.step_desc[j] = cp.step_desc[0];
      continue;
    }
    const long long o1 = chunk_off(k);
    long long lbo = 16;
    if (k + 16 < taps * cg) lbo = chunk_off(k + 16) - o1;
    if (lbo <= 0 || (lbo % 16) || lbo >= (1 << 18) || o1 >= (1 << 18)) return W4A8_ERR_UNSUPPORTED;
    cp.step_desc[j] = make_smem_desc(uint32_t(o1), uint32_t(lbo), sbo, cp.a_layout);
  }

  const int sms = device_sms();
  const int bn = g->o <= 64 ? 64 : (g->o <= 128 ? 128 : 256);
  p.M = 0;
  p.N = g->o;
  p.num_kb = groups * kbpg;
  p.tiles_m = cp.pack2 ? (g->n + 1) / 2 : g->n * cp.tiles_h * cp.tiles_w;
  p.tiles_n = (g->o + bn - 1) / bn;
  p.a_stage_bytes = 0;
  p.b_stage_bytes = bn * kBK;
  p.bp_stage_bytes = 0;
  const uint32_t per_stage = p.b_stage_bytes;
  // Resident weights: with a single n-tile and all k-blocks fitting next to
  // at least two halo stages, the CTA loads and unpacks the weights once and
  // then streams only input halos.
  const uint32_t bres_bytes = uint32_t(p.num_kb) * per_stage;
  // The epilogue's shared-memory copies of alpha and beta (not with the pool,
  // whose threads each hold their channel's pair in registers).
  cp.ab_pitch = (g->o + 15) & ~15;
  const uint32_t ab_bytes = (!g->pool && (epi->alpha || epi->beta) && g->o <= 1024)
                                ? (uint32_t(8 * cp.ab_pitch) + 1023u) & ~1023u
                                : 0u;
  // The pooled conv stages each epilogue set's pooled outputs for vector stores.
  const uint32_t pool_bytes = g->pool ? 4u * kPoolStageBytes : 0u;
  const uint32_t fixed_bytes = ab_bytes + pool_bytes;
  const int budget = kSmemBudget - int(fixed_bytes);
  // Resident weights also keep the MMA's descriptor table: one 16-byte (A, B)
  // pair per issued K-step, channel group and halo stage.
  const int gsteps = (kbpg - 1) * (kBK / 32) + cp.tail_steps;
  if (g->pool && groups != 1) return W4A8_ERR_UNSUPPORTED;  // the pooled conv: one channel group
  const uint32_t tab_stage = uint32_t((g->pool ? 2 : groups) * gsteps * 16);
  uint32_t dtab_bytes = 0;
  p.b_resident = 0;
  if (p.tiles_n == 1 && bres_bytes + 2 * (cp.halo_bytes + tab_stage) + 1024u <= uint32_t(budget)) {
    p.b_resident = 1;
    cp.extra_set = (bn == 64 && !g->pool) ? 1 : 0;  // the unpack warps drain a fifth buffer
    p.stages = 1;
    p.halo_stages = std::min<int>(kMaxHaloStages, (budget - 1024 - bres_bytes) / (cp.halo_bytes + tab_stage));
    dtab_bytes = (uint32_t(p.halo_stages) * tab_stage + 1023u) & ~1023u;
    p.bres_tx_bytes = i4 ? bres_bytes / 2 : bres_bytes;
  } else {
    if (g->pool) return W4A8_ERR_UNSUPPORTED;  // the pooled conv keeps its weights resident
    // Deepest halo pipeline (each stage is one tile's input window) that
    // still leaves at least three weight stages.
    p.stages = 0;
    for (int hs = 6; hs >= 1 && p.stages < 3; --hs) {
      p.halo_stages = hs;
      p.stages = pick_stages(per_stage, hs * cp.halo_bytes + fixed_bytes);
    }
    if (p.stages < 2) return W4A8_ERR_UNSUPPORTED;
  }
  p.a_off = 0;
  p.h_off = 0;
  const uint32_t halo_end = uint32_t(p.halo_stages) * cp.halo_bytes;
  cp.ab_off = ab_bytes ? halo_end : 0u;
  cp.pool_off = halo_end + ab_bytes;
  cp.dtab_off = halo_end + ab_bytes + pool_bytes;
  p.b_off = cp.dtab_off + dtab_bytes;
  p.bp_off = 0;
  p.tx_bytes = i4 ? p.b_stage_bytes / 2 : p.b_stage_bytes;
  p.tmem_cols = 2 * bn;
  p.err = device_error_word();
  if (!p.err) return W4A8_ERR_LAUNCH;
  fill_epi(p.epi, epi, out, g->o);
  p.epi.acc_fits_22 = (double)k_total * 128.0 * (i4 ? 8.0 : 128.0) < 4194304.0;
  if (g->out_layout == W4A8_LAYOUT_NHWC) {
    p.epi.s_img = (long long)g->ho * g->wo * g->ldo;
    p.epi.s_pix = g->ldo;
    p.epi.s_ch = 1;
  } else {
    p.epi.s_img = (long long)g->o * g->ho * g->wo;
    p.epi.s_pix = 1;
    p.epi.s_ch = (long long)g->ho * g->wo;
  }
  set_vec16(p.epi);

  CUtensorMap tA, tW, tH[4];
  std::memset(&tA, 0, sizeof(tA));
  std::memset(tH, 0, sizeof(tH));
  {
    const uint64_t dims[2] = {uint64_t(i4 ? k_total / 2 : k_total), uint64_t(g->o)};
    const uint64_t str[1] = {uint64_t(ldw)};
    const uint32_t box[2] = {uint32_t(i4 ? kBK / 2 : kBK), uint32_t(bn)};
    if (encode_u8(&tW, W, 2, dims, str, box, i4 ? CU_TENSOR_MAP_SWIZZLE_NONE : CU_TENSOR_MAP_SWIZZLE_128B))
      return W4A8_ERR_TENSORMAP;
  }
  const CUtensorMapSwizzle swz = cg == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                 : cg == 64  ? CU_TENSOR_MAP_SWIZZLE_64B
                                 : cg == 32  ? CU_TENSOR_MAP_SWIZZLE_32B
                                             : CU_TENSOR_MAP_SWIZZLE_NONE;
  for (int sl = 0; sl < ns; ++sl) {
    const int py = slot_py[sl], px = slot_px[sl];
    const int8_t* base = x + ((long long)py * g->w + px) * g->c;
    // (channels of the group, group, W, H, N); stride phases double W/H strides.
    // Two-image tiles order the dims (c, group, W, N, H): one box then lands
    // the two images' halo rows interleaved.
    const uint64_t wd = uint64_t((g->w - px + s - 1) / s), hd = uint64_t((g->h - py + s - 1) / s);
    const uint64_t ws = uint64_t(s) * g->c, hs = uint64_t(s) * g->w * g->c, ns_ = uint64_t(g->h) * g->w * g->c;
    const uint64_t dims[5] = {uint64_t(cg), uint64_t(groups), wd, cp.pack2 ? uint64_t(g->n) : hd,
                              cp.pack2 ? hd : uint64_t(g->n)};
    const uint64_t str[4] = {uint64_t(cg), ws, cp.pack2 ? ns_ : hs, cp.pack2 ? hs : ns_};
    const uint32_t box[5] = {uint32_t(cg), 1, uint32_t(cp.halo_w), cp.pack2 ? 2u : uint32_t(cp.halo_h),
                             cp.pack2 ? uint32_t(cp.halo_h) : 1u};
    if (cp.wc_bytes) {
      // 16-byte pixels at stride 1: (W * C, 1, 1, H, N), one box row per halo row.
      const uint64_t wc = uint64_t(g->w) * g->c;
      const uint64_t mdims[5] = {wc, 1, 1, uint64_t(g->h), uint64_t(g->n)};
      const uint64_t mstr[4] = {wc, wc, wc, uint64_t(g->h) * wc};
      const uint32_t mbox[5] = {uint32_t(cp.halo_w * g->c), 1, 1, uint32_t(cp.halo_h), 1};
      if (encode_u8(&tH[sl], base, 5, mdims, mstr, mbox, swz)) return W4A8_ERR_TENSORMAP;
      continue;
    }
    if (encode_u8(&tH[sl], base, 5, dims, str, box, swz)) return W4A8_ERR_TENSORMAP;
  }
  const int grid = std::min(p.tiles_m * p.tiles_n, sms);
  if (g->pool) return launch_t<64, false, true, true>(tA, tW, tH, p, grid, static_cast<cudaStream_t>(stream));
  return launch(i4, true, bn, tA, tW, tH, p, grid, static_cast<cudaStream_t>(stream));
}
