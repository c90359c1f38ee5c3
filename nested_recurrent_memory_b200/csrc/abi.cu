// extern "C" entry points of libngdn2: validation, workspace layout, path
// selection and launches. See include/ngdn2.h for the contract.

#include <string.h>

#include "fwd_params.cuh"

namespace ngdn2 {
cudaError_t launch_fwd_simt(const FwdParams& p, int stage, cudaStream_t stream);
int num_launches_simt(const FwdParams& p);
cudaError_t launch_update_simt(const UpdParams& u, cudaStream_t stream);
int64_t bwd_workspace_floats(const FwdParams& f);
int num_launches_bwd(const FwdParams& f);
struct BwdParams;
cudaError_t launch_update_bwd(const UpdBwdParams& u, cudaStream_t stream);
cudaError_t launch_bwd_abi(const ngdn2_bwd_args* a, const FwdParams& f, cudaStream_t stream);
}  // namespace ngdn2

#include "tc_api.cuh"

using namespace ngdn2;

namespace {

bool is_pow2(int x) { return x > 0 && (x & (x - 1)) == 0; }
bool dtype_ok(int d) { return d == NGDN2_F32 || d == NGDN2_BF16 || d == NGDN2_F16; }
bool dim_ok(int d) { return d >= 16 && d <= 128 && d % 16 == 0; }

int validate_fwd(const ngdn2_fwd_args* a, bool outputs = true) {
  if (!a) return NGDN2_ERR_NULL;
  if (a->abi_version != NGDN2_ABI_VERSION) return NGDN2_ERR_ABI;
  if (a->chunk_size != NGDN2_CHUNK) return NGDN2_ERR_CHUNK_SIZE;
  if (!dtype_ok(a->dtype) || !dtype_ok(a->param_dtype) || !dtype_ok(a->q_dtype) ||
      !dtype_ok(a->k_dtype) || !dtype_ok(a->v_dtype) || !dtype_ok(a->g_dtype) ||
      !dtype_ok(a->b_dtype) || !dtype_ok(a->w_dtype) || !dtype_ok(a->mix_dtype))
    return NGDN2_ERR_DTYPE;
  if (a->B < 1 || a->T < 0 || a->H < 1 || a->L < 1 || a->L > NGDN2_MAX_LEVELS)
    return NGDN2_ERR_SHAPE;
  if (!dim_ok(a->K) || !dim_ok(a->V)) return NGDN2_ERR_SHAPE;
  if (a->promotion != NGDN2_PROMOTION_LEARNED && a->promotion != NGDN2_PROMOTION_MERGE)
    return NGDN2_ERR_SHAPE;
  if (a->path < NGDN2_PATH_AUTO || a->path > NGDN2_PATH_TC_SEG) return NGDN2_ERR_SHAPE;
  for (int l = 0; l < a->L; ++l)
    if (a->firing[l] < 1) return NGDN2_ERR_FIRING;
  for (int l = 1; l < a->L; ++l) {
    // Pairs per firing feed the update scan, which needs a power of two
    // >= 16 (update_fwd.py:162-163); merge writes K pairs (probe.py:127).
    const int n = a->promotion == NGDN2_PROMOTION_MERGE ? a->K : a->n_queries[l - 1];
    if (n < 16 || !is_pow2(n)) return NGDN2_ERR_N_POW2;
    if (a->promotion == NGDN2_PROMOTION_LEARNED && (n > a->n_max || n > 128))
      return NGDN2_ERR_SHAPE;
  }
  if (!a->q || !a->k || !a->v || !a->g || !a->b || !a->w || !a->mix)
    return NGDN2_ERR_NULL;
  if (outputs && (!a->o || !a->final_state)) return NGDN2_ERR_NULL;
  if (a->L > 1 && (!a->query_banks || !a->key_projections || !a->b_projections ||
                   !a->w_projections || !a->g_projections))
    return NGDN2_ERR_NULL;
  if (a->gate && !a->status) return NGDN2_ERR_NULL;
  return NGDN2_OK;
}

// The start gate (ngdn2_fwd_args.gate): one thread polls the word, sleeping
// briefly between polls, and gives up after ``polls`` polls (0: 2^24, about
// a second), setting NGDN2_STATUS_GATE_TIMEOUT; every later kernel of the
// forward then returns at once (gate_closed).
__global__ void gate_kernel(const volatile int32_t* gate, uint32_t polls, int32_t* status) {
  const uint32_t n = polls ? polls : (1u << 24);
  for (uint32_t i = 0; i < n; ++i) {
    if (*gate != 0) return;
    __nanosleep(64);
  }
  atomicOr(status, NGDN2_STATUS_GATE_TIMEOUT);
}

void fill_params(const ngdn2_fwd_args* a, FwdParams* p) {
  memset(p, 0, sizeof(*p));
  p->B = a->B; p->T = a->T; p->H = a->H; p->K = a->K; p->V = a->V; p->L = a->L;
  p->NT = (a->T + NGDN2_CHUNK - 1) / NGDN2_CHUNK;
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
  p->q = QView{a->q, a->q_dtype, a->q_stride[0], a->q_stride[1], a->q_stride[2], a->q_stride[3], a->q_stride[4]};
  p->k = TokView{a->k, a->k_dtype, a->k_stride[0], a->k_stride[1], a->k_stride[2], a->k_stride[3]};
  p->v = TokView{a->v, a->v_dtype, a->v_stride[0], a->v_stride[1], a->v_stride[2], a->v_stride[3]};
  p->g = TokView{a->g, a->g_dtype, a->g_stride[0], a->g_stride[1], a->g_stride[2], a->g_stride[3]};
  p->b = TokView{a->b, a->b_dtype, a->b_stride[0], a->b_stride[1], a->b_stride[2], a->b_stride[3]};
  p->w = TokView{a->w, a->w_dtype, a->w_stride[0], a->w_stride[1], a->w_stride[2], a->w_stride[3]};
  p->mix = TokView{a->mix, a->mix_dtype, a->mix_stride[0], a->mix_stride[1], a->mix_stride[2], a->mix_stride[3]};
  p->raw_params[0] = a->query_banks;
  p->raw_params[1] = a->key_projections;
  p->raw_params[2] = a->b_projections;
  p->raw_params[3] = a->w_projections;
  p->raw_params[4] = a->g_projections;
  p->init = a->initial_state;
  p->o = a->o;
  p->fin = a->final_state;
  p->status = a->status;
  p->pl = ParamLayout::make(a->L, a->H, a->n_max, a->K, a->V);
  p->rec = ChunkRecord::make(a->K, a->V, a->L);
  p->ss = ScanScratch::make(a->K, a->V, np);
}

// (batch, head) pairs from which the fused family's one scan CTA per pair
// keeps enough SMs busy; below it the segmented family splits each level's
// sequence instead.
constexpr int kFusedMinPairs = 64;

int select_path(const ngdn2_fwd_args* a) {
  const bool tc_ok = tc_supports(a), seg_ok = seg_supports(a);
  if (a->path == NGDN2_PATH_SIMT) return NGDN2_PATH_SIMT;
  if (a->path == NGDN2_PATH_TC) return tc_ok ? int(NGDN2_PATH_TC) : int(NGDN2_ERR_UNSUPPORTED);
  if (a->path == NGDN2_PATH_TC_SEG)
    return seg_ok ? int(NGDN2_PATH_TC_SEG) : int(NGDN2_ERR_UNSUPPORTED);
  if (tc_ok && a->B * a->H >= kFusedMinPairs) return NGDN2_PATH_TC;
  if (seg_ok) return NGDN2_PATH_TC_SEG;
  return NGDN2_PATH_SIMT;
}

// Workspace of the SIMT path in floats: converted parameters, the chunk
// records and the per-(b, h) scan scratch.
int64_t simt_workspace_floats(const FwdParams& p) {
  return p.pl.size + int64_t(p.B) * p.H * p.NT * p.rec.size + int64_t(p.B) * p.H * p.ss.size;
}

}  // namespace

extern "C" {

int ngdn2_abi_version(void) { return NGDN2_ABI_VERSION; }
size_t ngdn2_sizeof_fwd_args(void) { return sizeof(ngdn2_fwd_args); }
size_t ngdn2_sizeof_update_args(void) { return sizeof(ngdn2_update_args); }

const char* ngdn2_error_string(int code) {
  switch (code) {
    case NGDN2_OK: return "ok";
    case NGDN2_ERR_CHUNK_SIZE: return "chunk_size must be 64";
    case NGDN2_ERR_N_POW2: return "pairs per firing must be a power of two >= 16";
    case NGDN2_ERR_BLOCK_V: return "block_v must be a power of two >= 16";
    case NGDN2_ERR_DIVISIBLE: return "V must be divisible by block_v";
    case NGDN2_ERR_UNIT_STRIDE: return "keys must be unit-stride along K";
    case NGDN2_ERR_INCONSISTENT: return "NF inconsistent with n_groups";
    case NGDN2_ERR_SHAPE: return "unsupported shape";
    case NGDN2_ERR_DTYPE: return "unsupported dtype";
    case NGDN2_ERR_NULL: return "a required pointer is NULL";
    case NGDN2_ERR_WORKSPACE: return "workspace too small";
    case NGDN2_ERR_UNSUPPORTED: return "the requested kernel path does not support this call";
    case NGDN2_ERR_CUDA: return "CUDA runtime error";
    case NGDN2_ERR_ABI: return "ABI version mismatch";
    case NGDN2_ERR_FIRING: return "firing intervals must be >= 1";
    default: return "unknown error";
  }
}

int ngdn2_fwd_select_path(const ngdn2_fwd_args* a) {
  const int rc = validate_fwd(a);
  return rc != NGDN2_OK ? rc : select_path(a);
}

int ngdn2_fwd_workspace_size(const ngdn2_fwd_args* a, size_t* bytes) {
  const int rc = validate_fwd(a);
  if (rc != NGDN2_OK) return rc;
  if (!bytes) return NGDN2_ERR_NULL;
  const int path = select_path(a);
  if (path < 0) return path;
  FwdParams p;
  fill_params(a, &p);
  if (path == NGDN2_PATH_TC) *bytes = tc_workspace_bytes(p);
  else if (path == NGDN2_PATH_TC_SEG) *bytes = seg_workspace_bytes(p);
  else *bytes = size_t(simt_workspace_floats(p)) * sizeof(float);
  return NGDN2_OK;
}

int ngdn2_fwd(const ngdn2_fwd_args* a, void* stream) { return ngdn2_fwd_stage(a, 0, stream); }

int ngdn2_fwd_num_launches(const ngdn2_fwd_args* a) {
  const int rc = validate_fwd(a);
  if (rc != NGDN2_OK) return rc;
  const int path = select_path(a);
  if (path < 0) return path;
  FwdParams p;
  fill_params(a, &p);
  return (a->gate ? 1 : 0) + (path == NGDN2_PATH_TC       ? num_launches_tc(p)
                               : path == NGDN2_PATH_TC_SEG ? num_launches_seg(p)
                                                           : num_launches_simt(p));
}

int ngdn2_fwd_stage(const ngdn2_fwd_args* a, int stage, void* stream) {
  if (stage < 0 || stage > 2) return NGDN2_ERR_SHAPE;
  const int rc = validate_fwd(a);
  if (rc != NGDN2_OK) return rc;
  const int path = select_path(a);
  if (path < 0) return path;
  FwdParams p;
  fill_params(a, &p);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t err;
  if (a->gate && (stage == 0 || stage == 1)) {
    gate_kernel<<<1, 1, 0, st>>>(a->gate, a->gate_polls, a->status);
    if (cudaGetLastError() != cudaSuccess) return NGDN2_ERR_CUDA;
  }
  if (path == NGDN2_PATH_TC) {
    const size_t need = tc_workspace_bytes(p);
    if (need > 0 && (!a->workspace || a->workspace_bytes < need)) return NGDN2_ERR_WORKSPACE;
    err = launch_fwd_tc(p, a->workspace, stage, st);
  } else if (path == NGDN2_PATH_TC_SEG) {
    const size_t need = seg_workspace_bytes(p);
    if (!a->workspace || a->workspace_bytes < need) return NGDN2_ERR_WORKSPACE;
    err = launch_fwd_seg(p, a->workspace, stage, st);
  } else {
    const size_t need = size_t(simt_workspace_floats(p)) * sizeof(float);
    if (!a->workspace || a->workspace_bytes < need) return NGDN2_ERR_WORKSPACE;
    float* ws = reinterpret_cast<float*>(a->workspace);
    p.params32 = ws;
    p.chunks = ws + p.pl.size;
    p.scan = p.chunks + int64_t(p.B) * p.H * p.NT * p.rec.size;
    err = launch_fwd_simt(p, stage, st);
  }
  return err == cudaSuccess ? NGDN2_OK : NGDN2_ERR_CUDA;
}

size_t ngdn2_sizeof_bwd_args(void) { return sizeof(ngdn2_bwd_args); }

// The backward's own checks on top of the forward's (its o, final_state,
// workspace and path are not used).
static int validate_bwd(const ngdn2_bwd_args* a) {
  if (!a) return NGDN2_ERR_NULL;
  if (a->abi_version != NGDN2_ABI_VERSION) return NGDN2_ERR_ABI;
  const int rc = validate_fwd(&a->fwd, false);
  if (rc != NGDN2_OK) return rc;
  if (!dtype_ok(a->d_o_dtype)) return NGDN2_ERR_DTYPE;
  if (!a->d_o || !a->dq || !a->dk || !a->dv || !a->dg || !a->db || !a->dw || !a->dmix)
    return NGDN2_ERR_NULL;
  return NGDN2_OK;
}

int ngdn2_bwd_workspace_size(const ngdn2_bwd_args* a, size_t* bytes) {
  const int rc = validate_bwd(a);
  if (rc != NGDN2_OK) return rc;
  if (!bytes) return NGDN2_ERR_NULL;
  FwdParams p;
  fill_params(&a->fwd, &p);
  *bytes = size_t(bwd_workspace_floats(p)) * sizeof(float);
  return NGDN2_OK;
}

int ngdn2_bwd_num_launches(const ngdn2_bwd_args* a) {
  const int rc = validate_bwd(a);
  if (rc != NGDN2_OK) return rc;
  FwdParams p;
  fill_params(&a->fwd, &p);
  return num_launches_bwd(p);
}

int ngdn2_bwd(const ngdn2_bwd_args* a, void* stream) {
  const int rc = validate_bwd(a);
  if (rc != NGDN2_OK) return rc;
  FwdParams p;
  fill_params(&a->fwd, &p);
  const size_t need = size_t(bwd_workspace_floats(p)) * sizeof(float);
  if (!a->workspace || a->workspace_bytes < need) return NGDN2_ERR_WORKSPACE;
  const cudaError_t err = launch_bwd_abi(a, p, reinterpret_cast<cudaStream_t>(stream));
  return err == cudaSuccess ? NGDN2_OK : NGDN2_ERR_CUDA;
}

size_t ngdn2_sizeof_update_bwd_args(void) { return sizeof(ngdn2_update_bwd_args); }

// update_bwd.py:197-206 -- the forward's checks, same order.
static int validate_update_bwd(const ngdn2_update_bwd_args* a) {
  if (!a) return NGDN2_ERR_NULL;
  if (a->abi_version != NGDN2_ABI_VERSION) return NGDN2_ERR_ABI;
  if (a->N < 16 || !is_pow2(a->N)) return NGDN2_ERR_N_POW2;
  if (a->block_v < 16 || !is_pow2(a->block_v)) return NGDN2_ERR_BLOCK_V;
  if (a->V % a->block_v) return NGDN2_ERR_DIVISIBLE;
  if (a->keys_stride[4] != 1) return NGDN2_ERR_UNIT_STRIDE;
  if (!(a->NG - 1 <= a->NF && a->NF <= a->NG)) return NGDN2_ERR_INCONSISTENT;
  if (!dtype_ok(a->dtype) || !dtype_ok(a->g_dtype)) return NGDN2_ERR_DTYPE;
  if (a->B < 1 || a->H < 1 || a->NF < 0 || a->NG < 1 || a->N > 128 || !dim_ok(a->K) ||
      !dim_ok(a->V))
    return NGDN2_ERR_SHAPE;
  if ((a->NF > 0 && (!a->keys || !a->values || !a->g || !a->b || !a->w || !a->dkeys ||
                     !a->dvalues || !a->dg || !a->db || !a->dw)) ||
      !a->states || !a->d_states || !a->d_final || (a->has_init && !a->dinit))
    return NGDN2_ERR_NULL;
  return NGDN2_OK;
}

static size_t update_bwd_bytes(const ngdn2_update_bwd_args* a) {
  const int64_t kv = int64_t(a->K) * a->V, nv = int64_t(a->N) * a->V;
  return sizeof(float) * size_t(a->B) * a->H * (align_floats(kv) * 3 + align_floats(nv) * 2);
}

int ngdn2_update_bwd_workspace_size(const ngdn2_update_bwd_args* a, size_t* bytes) {
  const int rc = validate_update_bwd(a);
  if (rc != NGDN2_OK) return rc;
  if (!bytes) return NGDN2_ERR_NULL;
  *bytes = update_bwd_bytes(a);
  return NGDN2_OK;
}

int ngdn2_update_state_bwd(const ngdn2_update_bwd_args* a, void* stream) {
  const int rc = validate_update_bwd(a);
  if (rc != NGDN2_OK) return rc;
  if (!a->workspace || a->workspace_bytes < update_bwd_bytes(a)) return NGDN2_ERR_WORKSPACE;
  UpdBwdParams u;
  u.B = a->B; u.NF = a->NF; u.NG = a->NG; u.H = a->H; u.K = a->K; u.V = a->V; u.N = a->N;
  u.dtype = a->dtype; u.g_dtype = a->g_dtype; u.has_init = a->has_init;
  u.states = a->states; u.keys = a->keys;
  u.skb = a->keys_stride[0]; u.skf = a->keys_stride[1]; u.skh = a->keys_stride[2];
  u.skn = a->keys_stride[3];
  u.values = a->values; u.g = a->g; u.b = a->b; u.w = a->w;
  u.d_states = a->d_states; u.d_final = a->d_final;
  u.dkeys = a->dkeys; u.dvalues = a->dvalues; u.dg = a->dg; u.db = a->db; u.dw = a->dw;
  u.dinit = a->dinit;
  u.scr = reinterpret_cast<float*>(a->workspace);
  const cudaError_t err = launch_update_bwd(u, reinterpret_cast<cudaStream_t>(stream));
  return err == cudaSuccess ? NGDN2_OK : NGDN2_ERR_CUDA;
}

// update_fwd.py:162-171 -- same checks, same order.
int ngdn2_update_state(const ngdn2_update_args* a, void* stream) {
  if (!a) return NGDN2_ERR_NULL;
  if (a->abi_version != NGDN2_ABI_VERSION) return NGDN2_ERR_ABI;
  if (a->N < 16 || !is_pow2(a->N)) return NGDN2_ERR_N_POW2;
  if (a->block_v < 16 || !is_pow2(a->block_v)) return NGDN2_ERR_BLOCK_V;
  if (a->V % a->block_v) return NGDN2_ERR_DIVISIBLE;
  if (a->keys_stride[4] != 1) return NGDN2_ERR_UNIT_STRIDE;
  if (!(a->NG - 1 <= a->NF && a->NF <= a->NG)) return NGDN2_ERR_INCONSISTENT;
  if (!dtype_ok(a->dtype) || !dtype_ok(a->g_dtype)) return NGDN2_ERR_DTYPE;
  if (a->B < 1 || a->H < 1 || a->NF < 0 || a->N > 128 || !dim_ok(a->K) || a->V < 16 ||
      a->V > 1024 || a->block_v > 128)
    return NGDN2_ERR_SHAPE;
  if ((a->NF > 0 && (!a->keys || !a->values || !a->g || !a->b || !a->w)) || !a->states ||
      !a->final_state)
    return NGDN2_ERR_NULL;
  UpdParams u;
  u.B = a->B; u.NF = a->NF; u.NG = a->NG; u.H = a->H; u.K = a->K; u.V = a->V; u.N = a->N;
  u.bv = a->block_v; u.dtype = a->dtype; u.g_dtype = a->g_dtype;
  u.keys = a->keys;
  u.skb = a->keys_stride[0]; u.skf = a->keys_stride[1]; u.skh = a->keys_stride[2];
  u.skn = a->keys_stride[3];
  u.values = a->values; u.g = a->g; u.b = a->b; u.w = a->w;
  u.init = a->initial_state; u.states = a->states; u.fin = a->final_state;
  const cudaError_t err = launch_update_simt(u, reinterpret_cast<cudaStream_t>(stream));
  return err == cudaSuccess ? NGDN2_OK : NGDN2_ERR_CUDA;
}

}  // extern "C"
