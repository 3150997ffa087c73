// Serving the batched MoE step: blind speculative decode and the per-row
// bookkeeping of a continuous-batching serve loop.
//
// Blind speculative decode (bench/dsv2_decode_bench.c
// :1110-1195 draft_prep / accept_commit, at batch 1 there): n_seq sequences
// of S rows each verify S tokens per step.  Device state per sequence i: the
// token stream ids[i][0..ctx) and its length len[i] = P + 1, P the index of
// the pending token (cache rows 0..P-1 committed).
//
//   sm100_spec_draft   cand[i][0] = ids[i][P]; cand[i][1..S) continue the most
//       recent earlier occurrence of the bigram (ids[P-1], ids[P]) inside
//       ids[0..P-1] (-1: a hole, never accepted), or, forced, the ids already
//       seeded at P + 1 ..; row i S + s gets token cand (a hole: the pending
//       token), cache slot i and position P + s.
//   sm100_spec_accept  k = the longest prefix with cand[s + 1] == am[s] (am:
//       the step's argmax per row); ids[P + 1 .. P + k] = cand[1 .. k],
//       ids[P + k + 1] = am[k] (the bonus token), len += k + 1.
//
// The verify rows run the base step's kernels row for row, so the committed
// stream is the base greedy stream; drafts only change how many positions a
// step commits.  A sequence whose next window would pass ctx is left as it is
// (no draft rows are written past the cache) and sets the status word.
//
//   sm100_serve_advance  after a step of B rows, each its own request (the
//       reference's serve loop, bench/dsv2_decode_bench.c:2760-2900, one
//       request at a time there): a row still inside its prompt takes the
//       prompt's next id (the step's argmax is dropped); otherwise the argmax
//       is appended to the row's output and the row stops at its eos id, its
//       max_new-th id or the end of the cache; the row's position advances.
#include "common.cuh"

using namespace sm100;

namespace {

constexpr int kSpecMaxS = 16;

__device__ uint32_t g_spec_status;

__global__ void __launch_bounds__(256) spec_draft_kernel(const int32_t *ids, const int32_t *len, int ctx, int S,
                                                         int forced, int32_t *tok, int32_t *cand, int32_t *row_pos,
                                                         int32_t *row_seq) {
  __shared__ int best;
  pdl_trigger();
  pdl_wait();
  const int i = blockIdx.x, t = threadIdx.x;
  const int32_t *id = ids + (int64_t)i * ctx;
  const int L = len[i], P = L - 1;
  const bool room = P >= 0 && P + S < ctx;   // rows P .. P + S - 1 inside the cache, ids up to P + S
  if (t == 0) {
    best = -1;
    if (!room) atomicOr(&g_spec_status, 1u);
  }
  __syncthreads();
  if (!room) {   // the window does not fit: the rows repeat the last step's pending token at P (clamped)
    const int pc = min(max(P, 0), ctx - 1);
    for (int s = t; s < S; s += blockDim.x) {
      tok[i * S + s] = id[pc];
      cand[i * S + s] = -1;
      row_pos[i * S + s] = pc;
      row_seq[i * S + s] = i;
    }
    return;
  }
  if (!forced && P >= 1) {
    const int a = id[P - 1], b = id[P];
    for (int j = t; j + 1 < P; j += blockDim.x)
      if (id[j] == a && id[j + 1] == b) atomicMax(&best, j);
  }
  __syncthreads();
  for (int s = t; s < S; s += blockDim.x) {
    int v;
    if (s == 0) v = id[P];
    else if (forced) v = P + s < ctx ? id[P + s] : -1;
    else v = best >= 0 && best + 1 + s <= P ? id[best + 1 + s] : -1;
    cand[i * S + s] = v;
    tok[i * S + s] = v >= 0 ? v : id[P];
    row_pos[i * S + s] = P + s;
    row_seq[i * S + s] = i;
  }
}

__global__ void spec_accept_kernel(int32_t *ids, int32_t *len, int ctx, int S, const int32_t *cand, const int32_t *am,
                                   unsigned long long *committed) {
  pdl_trigger();
  pdl_wait();
  const int i = blockIdx.x;
  if (threadIdx.x != 0) return;
  int32_t *id = ids + (int64_t)i * ctx;
  const int L = len[i], P = L - 1;
  if (P < 0 || P + S >= ctx) return;   // the draft left this sequence as it was
  const int32_t *c = cand + i * S, *a = am + i * S;
  int k = 0;
  while (k < S - 1 && c[k + 1] >= 0 && c[k + 1] == a[k]) k++;
  for (int j = 0; j < k; j++) id[P + 1 + j] = c[1 + j];
  id[P + 1 + k] = a[k];
  len[i] = P + k + 2;
  if (committed) atomicAdd(committed, (unsigned long long)(k + 1));
}

__global__ void serve_advance_kernel(int32_t *row_pos, int32_t *tok, const int32_t *am, const int32_t *prompt,
                                     const int32_t *plen, int32_t *out, int32_t *n_out, const int32_t *max_new,
                                     const int32_t *eos, int32_t *active, int B, int ctx) {
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B || !active[b]) return;
  const int p = row_pos[b];
  int nxt;
  if (p + 1 < plen[b] && p + 1 < ctx) {
    nxt = prompt[(int64_t)b * ctx + p + 1];
  } else {
    nxt = am[b];
    const int o = n_out[b];
    if (o >= 0 && o < ctx) out[(int64_t)b * ctx + o] = nxt;
    n_out[b] = o + 1;
    if (nxt == eos[b] || o + 1 >= max_new[b] || p + 2 >= ctx) {   // done: the slot idles at position 0
      active[b] = 0;
      row_pos[b] = 0;
      tok[b] = 0;
      return;
    }
  }
  row_pos[b] = p + 1;
  tok[b] = nxt;
}

}  // namespace

extern "C" int sm100_spec_draft(const int32_t *ids, const int32_t *len, int32_t n_seq, int32_t ctx, int32_t S,
                                int32_t forced, int32_t *tok, int32_t *cand, int32_t *row_pos, int32_t *row_seq,
                                void *stream) {
  if (!ids || !len || !tok || !cand || !row_pos || !row_seq || n_seq < 1 || S < 1 || S > kSpecMaxS || ctx < S + 1)
    return sm100_set_error(SM100_ERR_ARG, "spec_draft: n_seq %d ctx %d S %d (1..%d)", n_seq, ctx, S, kSpecMaxS);
  const cudaError_t e = launch_pdl(spec_draft_kernel, dim3(n_seq), dim3(256), 0, (cudaStream_t)stream, ids, len, ctx,
                                   S, forced, tok, cand, row_pos, row_seq);
  if (e != cudaSuccess) return sm100_set_error(SM100_ERR_CUDA, "spec_draft: %s", cudaGetErrorString(e));
  return launch_status("spec_draft");
}

extern "C" int sm100_spec_accept(int32_t *ids, int32_t *len, int32_t n_seq, int32_t ctx, int32_t S,
                                 const int32_t *cand, const int32_t *am, uint64_t *committed, void *stream) {
  if (!ids || !len || !cand || !am || n_seq < 1 || S < 1 || S > kSpecMaxS || ctx < S + 1)
    return sm100_set_error(SM100_ERR_ARG, "spec_accept: n_seq %d ctx %d S %d (1..%d)", n_seq, ctx, S, kSpecMaxS);
  const cudaError_t e = launch_pdl(spec_accept_kernel, dim3(n_seq), dim3(32), 0, (cudaStream_t)stream, ids, len, ctx,
                                   S, cand, am, reinterpret_cast<unsigned long long *>(committed));
  if (e != cudaSuccess) return sm100_set_error(SM100_ERR_CUDA, "spec_accept: %s", cudaGetErrorString(e));
  return launch_status("spec_accept");
}

extern "C" int sm100_serve_advance(int32_t *row_pos, int32_t *tok, const int32_t *am, const int32_t *prompt,
                                   const int32_t *plen, int32_t *out, int32_t *n_out, const int32_t *max_new,
                                   const int32_t *eos, int32_t *active, int32_t B, int32_t ctx, void *stream) {
  if (!row_pos || !tok || !am || !prompt || !plen || !out || !n_out || !max_new || !eos || !active || B < 1 ||
      ctx < 2)
    return sm100_set_error(SM100_ERR_ARG, "serve_advance: B %d ctx %d", B, ctx);
  const cudaError_t e = launch_pdl(serve_advance_kernel, dim3((B + 127) / 128), dim3(128), 0, (cudaStream_t)stream,
                                   row_pos, tok, am, prompt, plen, out, n_out, max_new, eos, active, B, ctx);
  if (e != cudaSuccess) return sm100_set_error(SM100_ERR_CUDA, "serve_advance: %s", cudaGetErrorString(e));
  return launch_status("serve_advance");
}

extern "C" uint32_t sm100_spec_status(void) {
  uint32_t v = 0, z = 0;
  cudaDeviceSynchronize();
  cudaMemcpyFromSymbol(&v, g_spec_status, sizeof(v));
  cudaMemcpyToSymbol(g_spec_status, &z, sizeof(z));
  return v;
}
