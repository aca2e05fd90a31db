// Parallel block decoding on device: row-wise argmax, the draft step (K7) and the verify / greedy
// accept / rollback step (K8). Reference: OrthrusLM.diffusion_generate
// (orthrus/modeling_orthrus.py:404-534) and decoding.decode / _verify / _advance
// (orthrus/decoding.py:336-429), greedy (temperature 0).
//
// The KV cache is a preallocated [B, Hkv, cap, D] buffer per layer with the committed length of
// sequence b in start[b]: rolling the cache back after a rejected draft is just writing the new
// length, positions past it are dead and are overwritten by the next verification. Nothing here
// synchronises with the host, so a whole draft + verify + accept cycle can be replayed as one CUDA
// graph; the host only polls the done flags now and then.
#pragma once

#include "sm100.cuh"

namespace orthrus {

// Argmax of one fp32 row, lowest index among equal maxima (torch.argmax semantics).
__device__ __forceinline__ void argmax_pair_merge(float& v, int64_t& i, float ov, int64_t oi) {
  if (ov > v || (ov == v && oi < i)) {
    v = ov;
    i = oi;
  }
}

template <int THREADS>
__device__ int64_t block_argmax_row(const float* __restrict__ row, int64_t V) {
  __shared__ float sv[THREADS / 32];
  __shared__ int64_t si[THREADS / 32];
  float best = -INFINITY;
  int64_t bi = INT64_MAX;
  const bool vec = (V % 4 == 0) && ((reinterpret_cast<uintptr_t>(row) & 15) == 0);
  if (vec) {
    const float4* r4 = reinterpret_cast<const float4*>(row);
    for (int64_t j = threadIdx.x; j < V / 4; j += THREADS) {
      const float4 x = r4[j];
      argmax_pair_merge(best, bi, x.x, 4 * j);
      argmax_pair_merge(best, bi, x.y, 4 * j + 1);
      argmax_pair_merge(best, bi, x.z, 4 * j + 2);
      argmax_pair_merge(best, bi, x.w, 4 * j + 3);
    }
  } else {
    for (int64_t j = threadIdx.x; j < V; j += THREADS) argmax_pair_merge(best, bi, row[j], j);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, off);
    const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, off);
    argmax_pair_merge(best, bi, ov, oi);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sv[warp] = best;
    si[warp] = bi;
  }
  __syncthreads();
  if (warp == 0) {
    best = lane < THREADS / 32 ? sv[lane] : -INFINITY;
    bi = lane < THREADS / 32 ? si[lane] : INT64_MAX;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, off);
      const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, off);
      argmax_pair_merge(best, bi, ov, oi);
    }
  }
  if (bi == INT64_MAX) bi = 0;  // all NaN / empty row
  return bi;
}

__global__ void __launch_bounds__(512) argmax_rows_kernel(const float* __restrict__ logits, int64_t ldl, int64_t V,
                                                          int64_t* __restrict__ out) {
  const int64_t r = blockIdx.x;
  const int64_t i = block_argmax_row<512>(logits + r * ldl, V);
  if (threadIdx.x == 0) out[r] = i;
}

// verify_ids[b] = [anchor[b], argmax(logits[b, 0]), ..., argmax(logits[b, K-2])]
__global__ void __launch_bounds__(512) decode_draft_kernel(const float* __restrict__ logits, int K, int64_t V,
                                                           const int64_t* __restrict__ anchor,
                                                           const uint8_t* __restrict__ done,
                                                           int64_t* __restrict__ verify_ids) {
  const int64_t b = blockIdx.y;
  const int i = blockIdx.x;  // draft position 0..K-2
  if (done && done[b]) return;
  const int64_t tok = block_argmax_row<512>(logits + (b * K + i) * V, V);
  if (threadIdx.x == 0) {
    verify_ids[b * K + 1 + i] = tok;
    if (i == 0) verify_ids[b * K] = anchor[b];
  }
}

// The same from the rows' argmax ids [B * K] (the LM head's argmax without logits).
__global__ void decode_draft_ids_kernel(const int64_t* __restrict__ ids, int64_t B, int K,
                                        const int64_t* __restrict__ anchor, const uint8_t* __restrict__ done,
                                        int64_t* __restrict__ verify_ids) {
  const int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (e >= B * K) return;
  const int64_t b = e / K;
  const int i = static_cast<int>(e % K);
  if (done && done[b]) return;
  verify_ids[e] = i == 0 ? anchor[b] : ids[b * K + i - 1];
}

__device__ __forceinline__ bool is_eos(int64_t tok, const int64_t* eos, int n_eos) {
  for (int i = 0; i < n_eos; ++i)
    if (eos[i] == tok) return true;
  return false;
}

// The end of a cycle of sequence b once its accepted drafts and bonus token are known: log the
// accepted count, append the kept drafts and the bonus token, stop at EOS or the length limit,
// and roll the cache back by writing the committed length (decoding._advance,
// orthrus/decoding.py:354-369).
__device__ inline void commit_cycle(int64_t b, int K, int accepted, int64_t bonus,
                                    const int64_t* __restrict__ verify_ids, const int64_t* __restrict__ eos,
                                    int n_eos, const int32_t* __restrict__ max_len, int32_t* __restrict__ start,
                                    int64_t* __restrict__ anchor, uint8_t* __restrict__ done,
                                    int64_t* __restrict__ out_tokens, int32_t* __restrict__ out_len, int64_t out_cap,
                                    int32_t* __restrict__ accepted_log, int32_t* __restrict__ cycle,
                                    int64_t log_cap) {
  const int st = start[b];
  const int ml = max_len[b];
  const int64_t* drafts = verify_ids + b * K + 1;
  const int c = cycle[b];
  if (c < log_cap) accepted_log[b * log_cap + c] = accepted;
  cycle[b] = c + 1;
  int n = out_len[b];
  int64_t* out = out_tokens + b * out_cap;
  for (int i = 0; i < accepted; ++i) {
    if (n < out_cap) out[n] = drafts[i];
    ++n;
    if (is_eos(drafts[i], eos, n_eos)) {
      out_len[b] = n;
      start[b] = st + i + 1;
      done[b] = 1;
      return;
    }
  }
  const int ns = st + accepted + 1;
  bool fin = false;
  if (ns < ml) {
    if (n < out_cap) out[n] = bonus;
    ++n;
    if (is_eos(bonus, eos, n_eos)) fin = true;
  }
  out_len[b] = n;
  start[b] = ns;
  anchor[b] = bonus;
  if (fin || ns >= ml - 1) done[b] = 1;
}

// One thread per sequence: greedy longest-prefix accept (stopping after an accepted EOS) and the
// AR token after it as the bonus (decoding._verify, orthrus/decoding.py:336-353), then the commit.
__global__ void decode_accept_kernel(int64_t B, int K, const int64_t* __restrict__ verify_ids,
                                     const int64_t* __restrict__ ar, const int64_t* __restrict__ eos, int n_eos,
                                     const int32_t* __restrict__ max_len, int32_t* __restrict__ start,
                                     int64_t* __restrict__ anchor, uint8_t* __restrict__ done,
                                     int64_t* __restrict__ out_tokens, int32_t* __restrict__ out_len,
                                     int64_t out_cap, int32_t* __restrict__ accepted_log, int32_t* __restrict__ cycle,
                                     int64_t log_cap) {
  const int64_t b = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (b >= B || done[b]) return;
  const int block_len = min(K, max_len[b] - start[b]);
  const int64_t* drafts = verify_ids + b * K + 1;
  const int64_t* pred = ar + b * K;
  int accepted = 0;
  while (accepted < block_len - 1 && drafts[accepted] == pred[accepted]) {
    ++accepted;
    if (is_eos(drafts[accepted - 1], eos, n_eos)) break;
  }
  commit_cycle(b, K, accepted, pred[accepted], verify_ids, eos, n_eos, max_len, start, anchor, done, out_tokens,
               out_len, out_cap, accepted_log, cycle, log_cap);
}

}  // namespace orthrus
