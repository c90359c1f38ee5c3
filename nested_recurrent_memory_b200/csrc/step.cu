// One-token decode step (nested_gdn2/ops/naive.py:42-134,
// naive_step_nested_gdn2), the path the layer takes past its chunked prefix
// (nested_gdn2.py:218-224). Level 0 takes the token's delta-rule write and
// every level is read with the token's query and mixed into o: the value
// columns are independent there, so a CTA takes one (b, h) and 16 or 32 of
// its columns (more CTAs in flight over the state). Then, when this token
// completes some row's firing, a second kernel (one CTA per (b, h))
// promotes each firing level bottom-up on the new state. fp32 arithmetic on
// CUDA cores: a step touches each state element once or twice, so it is
// bound by the state traffic.

#include <string.h>

#include "fwd_params.cuh"
#include "promote_simt.cuh"

namespace ngdn2 {
cudaError_t launch_convert_params(const FwdParams& p, cudaStream_t stream);
}  // namespace ngdn2

using namespace ngdn2;

namespace {

constexpr int kStepThreads = 256;

// Columns of V per CTA of the write / read kernel.
__host__ __device__ inline int step_cols(int V) { return V % 32 == 0 ? 32 : 16; }

// S' = e^g S - k (k b e^g)^T S + k (v w)^T for one pair (naive.py:7-39,
// with N = 1) and the reads sum_l mix_l scale q_l S_l (naive.py:111-113),
// for the columns [c0, c0 + step_cols(V)) of one (b, h).
__global__ void __launch_bounds__(kStepThreads)
step_kernel(FwdParams p, const float* Sin, float* Sout) {
  __shared__ float eg[128], kv[128], kbe[128], vw[128], mixv[NGDN2_MAX_LEVELS];
  __shared__ float sq[NGDN2_MAX_LEVELS][128];
  __shared__ float red[kStepThreads];
  const int bh = blockIdx.x, b = bh / p.H, h = bh % p.H;
  const int K = p.K, V = p.V, L = p.L, tid = threadIdx.x;
  const int Vs = step_cols(V), c0 = blockIdx.y * Vs;
  const int64_t lv = int64_t(K) * V;
  const float* S = Sin + int64_t(bh) * L * lv;
  float* So = Sout + int64_t(bh) * L * lv;

  for (int d = tid; d < K; d += blockDim.x) {
    const float kk = p.k.at(b, 0, h, d), e = expf(p.g.at(b, 0, h, d));
    eg[d] = e;
    kv[d] = kk;
    kbe[d] = kk * p.b.at(b, 0, h, d) * e;
    for (int l = 0; l < L; ++l) sq[l][d] = p.scale * p.q.at(b, 0, h, l, d);
  }
  for (int cl = tid; cl < Vs; cl += blockDim.x)
    vw[cl] = p.v.at(b, 0, h, c0 + cl) * p.w.at(b, 0, h, c0 + cl);
  if (tid < L) mixv[tid] = p.mix.at(b, 0, h, tid);
  __syncthreads();

  // Thread (cl, s): column c0 + cl, rows s, s + sp, ... (sp slices).
  const int sp = kStepThreads / Vs, cl = tid % Vs, s = tid / Vs, c = c0 + cl;
  auto reduce = [&](float part) {
    __syncthreads();
    red[s * Vs + cl] = part;
    __syncthreads();
    float t = 0.f;
    for (int j = 0; j < sp; ++j) t += red[j * Vs + cl];
    return t;
  };
  // Level 0: d_c = sum_k (k b e^g)_k S[k][c], then the write and its read.
  float part = 0.f;
  for (int k = s; k < K; k += sp) part = fmaf(kbe[k], S[int64_t(k) * V + c], part);
  const float dc = reduce(part);
  part = 0.f;
  {
    const float u = vw[cl] - dc;
    for (int k = s; k < K; k += sp) {
      const float x = fmaf(eg[k], S[int64_t(k) * V + c], kv[k] * u);
      So[int64_t(k) * V + c] = x;
      part = fmaf(sq[0][k], x, part);
    }
  }
  float o = mixv[0] * reduce(part);
  // Upper levels: read (the state before any promotion of this token).
  for (int l = 1; l < L; ++l) {
    part = 0.f;
    const float* Sl = S + l * lv;
    float* Sol = So + l * lv;
    for (int k = s; k < K; k += sp) {
      const float x = Sl[int64_t(k) * V + c];
      if (Sol != Sl) Sol[int64_t(k) * V + c] = x;
      part = fmaf(sq[l][k], x, part);
    }
    o = fmaf(mixv[l], reduce(part), o);
  }
  if (s == 0) store_elem(p.o, int64_t(bh) * V + c, o, p.dtype);
}

// The promotions of a row whose token completes a firing, bottom-up, on
// the new state (naive.py:115-132).
__global__ void __launch_bounds__(kStepThreads)
step_promote_kernel(FwdParams p, const int64_t* positions, int64_t position, int chunk,
                    float* Sout) {
  __shared__ float gsm[kGemmSmemFloats];
  const int bh = blockIdx.x, b = bh / p.H, h = bh % p.H;
  const int64_t lv = int64_t(p.K) * p.V;
  float* So = Sout + int64_t(bh) * p.L * lv;
  const int64_t end = (positions ? positions[b] : position) + 1;
  if (p.L < 2 || end % chunk != 0) return;
  const int64_t ch = end / chunk;
  float* sc = p.scan + int64_t(bh) * p.ss.size;
  for (int l = 1; l < p.L; ++l) {
    if (ch % p.firing[l] != 0) continue;
    promote_simt(p, b, h, l, So, sc, gsm);
    __syncthreads();
  }
}

bool is_pow2(int x) { return x > 0 && (x & (x - 1)) == 0; }
bool dtype_ok(int d) { return d == NGDN2_F32 || d == NGDN2_BF16 || d == NGDN2_F16; }
bool dim_ok(int d) { return d >= 16 && d <= 128 && d % 16 == 0; }

int validate_step(const ngdn2_step_args* a) {
  if (!a) return NGDN2_ERR_NULL;
  if (a->abi_version != NGDN2_ABI_VERSION) return NGDN2_ERR_ABI;
  if (a->chunk_size < 1) return NGDN2_ERR_SHAPE;
  if (!dtype_ok(a->dtype) || !dtype_ok(a->param_dtype) || !dtype_ok(a->q_dtype) ||
      !dtype_ok(a->k_dtype) || !dtype_ok(a->v_dtype) || !dtype_ok(a->g_dtype) ||
      !dtype_ok(a->b_dtype) || !dtype_ok(a->w_dtype) || !dtype_ok(a->mix_dtype))
    return NGDN2_ERR_DTYPE;
  if (a->B < 1 || a->H < 1 || a->L < 1 || a->L > NGDN2_MAX_LEVELS) return NGDN2_ERR_SHAPE;
  if (!dim_ok(a->K) || !dim_ok(a->V)) return NGDN2_ERR_SHAPE;
  if (a->promotion != NGDN2_PROMOTION_LEARNED && a->promotion != NGDN2_PROMOTION_MERGE)
    return NGDN2_ERR_SHAPE;
  for (int l = 0; l < a->L; ++l)
    if (a->firing[l] < 1) return NGDN2_ERR_FIRING;
  for (int l = 1; l < a->L; ++l) {
    const int n = a->promotion == NGDN2_PROMOTION_MERGE ? a->K : a->n_queries[l - 1];
    if (n < 16 || !is_pow2(n)) return NGDN2_ERR_N_POW2;
    if (a->promotion == NGDN2_PROMOTION_LEARNED && (n > a->n_max || n > 128))
      return NGDN2_ERR_SHAPE;
  }
  if (!a->q || !a->k || !a->v || !a->g || !a->b || !a->w || !a->mix || !a->o || !a->state_in ||
      !a->state_out)
    return NGDN2_ERR_NULL;
  if (a->L > 1 && (!a->query_banks || !a->key_projections || !a->b_projections ||
                   !a->w_projections || !a->g_projections))
    return NGDN2_ERR_NULL;
  return NGDN2_OK;
}

// The step as a one-token forward: views without a T dimension (stride 0).
void fill_step_params(const ngdn2_step_args* a, FwdParams* p) {
  memset(p, 0, sizeof(*p));
  p->B = a->B; p->T = 1; p->H = a->H; p->K = a->K; p->V = a->V; p->L = a->L; p->NT = 1;
  p->n_max = a->n_max; p->promotion = a->promotion;
  p->dtype = a->dtype; p->param_dtype = a->param_dtype; p->scale = a->scale;
  int np = 16;
  for (int l = 0; l < NGDN2_MAX_LEVELS; ++l) {
    p->firing[l] = l < a->L ? a->firing[l] : 1;
    p->nq[l] = a->n_queries[l];
    if (l + 1 < a->L) {
      const int n = a->promotion == NGDN2_PROMOTION_MERGE ? a->K : a->n_queries[l];
      if (n > np) np = n;
    }
  }
  p->NP = np;
  p->q = QView{a->q, a->q_dtype, a->q_stride[0], 0, a->q_stride[1], a->q_stride[2], a->q_stride[3]};
  p->k = TokView{a->k, a->k_dtype, a->k_stride[0], 0, a->k_stride[1], a->k_stride[2]};
  p->v = TokView{a->v, a->v_dtype, a->v_stride[0], 0, a->v_stride[1], a->v_stride[2]};
  p->g = TokView{a->g, a->g_dtype, a->g_stride[0], 0, a->g_stride[1], a->g_stride[2]};
  p->b = TokView{a->b, a->b_dtype, a->b_stride[0], 0, a->b_stride[1], a->b_stride[2]};
  p->w = TokView{a->w, a->w_dtype, a->w_stride[0], 0, a->w_stride[1], a->w_stride[2]};
  p->mix = TokView{a->mix, a->mix_dtype, a->mix_stride[0], 0, a->mix_stride[1], a->mix_stride[2]};
  p->raw_params[0] = a->query_banks;
  p->raw_params[1] = a->key_projections;
  p->raw_params[2] = a->b_projections;
  p->raw_params[3] = a->w_projections;
  p->raw_params[4] = a->g_projections;
  p->o = a->o;
  p->status = a->status;
  p->pl = ParamLayout::make(a->L, a->H, a->n_max, a->K, a->V);
  p->ss = ScanScratch::make(a->K, a->V, np);
}

int64_t step_workspace_floats(const FwdParams& p) {
  return p.L > 1 ? p.pl.size + int64_t(p.B) * p.H * p.ss.size : 0;
}

}  // namespace

extern "C" {

NGDN2_API size_t ngdn2_sizeof_step_args(void) { return sizeof(ngdn2_step_args); }

NGDN2_API int ngdn2_step_workspace_size(const ngdn2_step_args* args, size_t* bytes) {
  const int rc = validate_step(args);
  if (rc != NGDN2_OK) return rc;
  if (!bytes) return NGDN2_ERR_NULL;
  FwdParams p;
  fill_step_params(args, &p);
  *bytes = size_t(step_workspace_floats(p)) * sizeof(float);
  return NGDN2_OK;
}

NGDN2_API int ngdn2_step(const ngdn2_step_args* args, void* stream) {
  const int rc = validate_step(args);
  if (rc != NGDN2_OK) return rc;
  FwdParams p;
  fill_step_params(args, &p);
  const size_t need = size_t(step_workspace_floats(p)) * sizeof(float);
  if (need > 0 && (!args->workspace || args->workspace_bytes < need)) return NGDN2_ERR_WORKSPACE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (p.L > 1) {
    float* ws = static_cast<float*>(args->workspace);
    p.params32 = ws;
    p.scan = ws + p.pl.size;
    // The fp32 parameter copy is needed only when some row can fire: with
    // one host-side position that is known here.
    bool may_fire = args->positions != nullptr;
    if (!may_fire && (args->position + 1) % args->chunk_size == 0) {
      const int64_t ch = (args->position + 1) / args->chunk_size;
      for (int l = 1; l < p.L; ++l) may_fire |= ch % p.firing[l] == 0;
    }
    if (may_fire && launch_convert_params(p, st) != cudaSuccess) return NGDN2_ERR_CUDA;
    step_kernel<<<dim3(p.B * p.H, p.V / step_cols(p.V)), kStepThreads, 0, st>>>(
        p, args->state_in, args->state_out);
    if (cudaGetLastError() != cudaSuccess) return NGDN2_ERR_CUDA;
    if (may_fire)
      step_promote_kernel<<<p.B * p.H, kStepThreads, 0, st>>>(p, args->positions, args->position,
                                                              args->chunk_size, args->state_out);
    return cudaGetLastError() == cudaSuccess ? NGDN2_OK : NGDN2_ERR_CUDA;
  }
  step_kernel<<<dim3(p.B * p.H, p.V / step_cols(p.V)), kStepThreads, 0, st>>>(
      p, args->state_in, args->state_out);
  return cudaGetLastError() == cudaSuccess ? NGDN2_OK : NGDN2_ERR_CUDA;
}

}  // extern "C"
