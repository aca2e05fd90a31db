// Sampled parallel block decoding on device: the sampling filter of diffusion_generate's `pick`
// (temperature, top-k, top-p; orthrus/modeling_orthrus.py:437-449) over each row's top
// candidates, the draft step, and exact rejection sampling of the drafts against the verify pass
// (orthrus/modeling_orthrus.py:498-511), ending in the same commit / rollback / EOS bookkeeping as
// the greedy cycle.
//
// Each row's distribution lives on its C top candidates (values sorted descending with their
// token ids): top-k keeps at most top_k of them plus ties at the k-th value, so C = top_k + a few
// holds it. Random numbers come from Philox4x32-10 (Salmon, Moraes, Dror and Shaw, "Parallel
// random numbers: as easy as 1, 2, 3", SC 2011) keyed by a per-decode seed and counted by
// (sequence, cycle, position, purpose): every draw is a pure function of the decode's state, so a
// cycle replays as a CUDA graph and a run is reproducible from its seed.
#pragma once

#include "decode.cuh"

namespace orthrus {

constexpr int kSampleMaxCand = 128;  // candidates per row (top_k + ties)
constexpr int kSampleMaxBlock = 64;  // block size K of a sampled cycle

enum SamplePurpose : uint32_t { kDrawDraft = 0, kDrawAccept = 1, kDrawBonus = 2, kDrawFirst = 3 };

struct Philox4 {
  uint32_t x, y, z, w;
};

// Philox4x32 with 10 rounds: multiply-high/low of counter words 0 and 2 by the round multipliers,
// xor the high halves into the other words with the key, and bump the key by the Weyl constants.
__host__ __device__ inline Philox4 philox4x32_10(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3, uint32_t k0,
                                                 uint32_t k1) {
  constexpr uint32_t kM0 = 0xD2511F53u, kM1 = 0xCD9E8D57u, kW0 = 0x9E3779B9u, kW1 = 0xBB67AE85u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint64_t p0 = static_cast<uint64_t>(kM0) * c0;
    const uint64_t p1 = static_cast<uint64_t>(kM1) * c2;
    const uint32_t hi0 = static_cast<uint32_t>(p0 >> 32), lo0 = static_cast<uint32_t>(p0);
    const uint32_t hi1 = static_cast<uint32_t>(p1 >> 32), lo1 = static_cast<uint32_t>(p1);
    c0 = hi1 ^ c1 ^ k0;
    c1 = lo1;
    c2 = hi0 ^ c3 ^ k1;
    c3 = lo0;
    k0 += kW0;
    k1 += kW1;
  }
  return {c0, c1, c2, c3};
}

// Uniform in [0, 1) with 24 random bits, for draw (sequence, cycle, position, purpose).
__device__ __forceinline__ float sample_uniform(uint64_t seed, uint32_t seq, uint32_t cycle, uint32_t pos,
                                                uint32_t purpose) {
  const Philox4 r = philox4x32_10(seq, cycle, pos, purpose, static_cast<uint32_t>(seed),
                                  static_cast<uint32_t>(seed >> 32));
  return static_cast<float>(r.x >> 8) * (1.0f / 16777216.0f);
}

// The filtered distribution of one row over its candidates (vals sorted descending): values
// divided by the temperature; those below the top_k-th dropped (ties kept); then the smallest
// descending prefix whose probability mass exceeds top_p kept (the first always); softmax over
// the rest. probs[j] = 0 for dropped candidates. Returns the number of candidates kept.
__device__ inline int sample_filter_row(const float* __restrict__ vals, int C, float temperature, int top_k,
                                        float top_p, float* __restrict__ probs) {
  float x[kSampleMaxCand];
  for (int j = 0; j < C; ++j) x[j] = vals[j] / temperature;
  int n = C;
  if (top_k > 0 && top_k < C) {
    const float kth = x[top_k - 1];
    n = top_k;
    while (n < C && x[n] >= kth) ++n;
  }
  const float m = x[0];
  float z = 0.f;
  for (int j = 0; j < n; ++j) {
    x[j] = expf(x[j] - m);
    z += x[j];
  }
  int keep = n;
  if (top_p < 1.f) {
    float cum = 0.f;
    for (int j = 0; j < n; ++j) {
      if (j > 0 && cum > top_p) {
        keep = j;
        break;
      }
      cum += x[j] / z;
    }
  }
  float z2 = 0.f;
  for (int j = 0; j < keep; ++j) z2 += x[j];
  const float inv = 1.f / z2;
  for (int j = 0; j < C; ++j) probs[j] = j < keep ? x[j] * inv : 0.f;
  return keep;
}

// Index of the candidate a uniform u picks from weights w[0..C) of total mass `total`: the first
// whose running sum exceeds u * total (the last positive one if rounding leaves none).
__device__ inline int sample_pick(const float* __restrict__ w, int C, float total, float u) {
  const float target = u * total;
  float cum = 0.f;
  int last = 0;
  for (int j = 0; j < C; ++j) {
    if (w[j] > 0.f) {
      cum += w[j];
      last = j;
      if (cum > target) return j;
    }
  }
  return last;
}

__device__ __forceinline__ float cand_prob(const int64_t* __restrict__ ids, const float* __restrict__ probs, int C,
                                           int64_t token) {
  for (int j = 0; j < C; ++j)
    if (ids[j] == token) return probs[j];
  return 0.f;
}

// probs [R, C] of candidate rows [R, C]; one thread per row.
__global__ void sample_probs_kernel(const float* __restrict__ vals, int64_t R, int C, float temperature, int top_k,
                                    float top_p, float* __restrict__ probs) {
  const int64_t r = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (r >= R) return;
  sample_filter_row(vals + r * C, C, temperature, top_k, top_p, probs + r * C);
}

// One token per candidate row (the prefill's first token of each sequence), draw (r, cycle, 0,
// kDrawFirst) with the cycle counter of row r (0 before any cycle).
__global__ void sample_rows_kernel(const float* __restrict__ vals, const int64_t* __restrict__ ids, int64_t R, int C,
                                   float temperature, int top_k, float top_p, uint64_t seed,
                                   const int32_t* __restrict__ cycle, int64_t* __restrict__ tokens) {
  const int64_t r = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (r >= R) return;
  float p[kSampleMaxCand];
  sample_filter_row(vals + r * C, C, temperature, top_k, top_p, p);
  float total = 0.f;
  for (int j = 0; j < C; ++j) total += p[j];
  const uint32_t cyc = cycle ? static_cast<uint32_t>(cycle[r]) : 0u;
  const float u = sample_uniform(seed, static_cast<uint32_t>(r), cyc, 0u, kDrawFirst);
  tokens[r] = ids[r * C + sample_pick(p, C, total, u)];
}

// Draft step of a sampled cycle: grid B, one thread per draft position i < K-1. The draft
// distribution q_i is kept in draft_probs [B, K-1, C] for the accept step.
__global__ void decode_sample_draft_kernel(const float* __restrict__ vals, const int64_t* __restrict__ ids, int K,
                                           int C, float temperature, int top_k, float top_p, uint64_t seed,
                                           const int32_t* __restrict__ cycle, const int64_t* __restrict__ anchor,
                                           const uint8_t* __restrict__ done, int64_t* __restrict__ verify_ids,
                                           float* __restrict__ draft_probs) {
  const int64_t b = blockIdx.x;
  const int i = threadIdx.x;
  if (done[b]) return;
  if (i == 0) verify_ids[b * K] = anchor[b];
  if (i >= K - 1) return;
  const int64_t row = b * (K - 1) + i;
  float* q = draft_probs + row * C;
  sample_filter_row(vals + row * C, C, temperature, top_k, top_p, q);
  float total = 0.f;
  for (int j = 0; j < C; ++j) total += q[j];
  const float u = sample_uniform(seed, static_cast<uint32_t>(b), static_cast<uint32_t>(cycle[b]),
                                 static_cast<uint32_t>(i), kDrawDraft);
  verify_ids[b * K + 1 + i] = ids[row * C + sample_pick(q, C, total, u)];
}

}  // namespace orthrus

namespace orthrus {

// Verify / accept step of a sampled cycle: grid B, one thread per block position (K <= 64).
// Thread i filters verify row i into p_i; draft i is kept while u_i < min(1, p_i(d_i) / q_i(d_i))
// (all positions test at once, each with its own draw; the first failure ends the accepted run,
// as the reference's sequential draws do). At the first rejection the bonus token comes from the
// normalised residual max(p - q, 0) (p itself when its mass is <= 1e-5), after a full accept from
// p of the next position. Then the greedy cycle's commit.
__global__ void __launch_bounds__(kSampleMaxBlock) decode_sample_accept_kernel(
    const float* __restrict__ vals, const int64_t* __restrict__ ids, const float* __restrict__ draft_probs,
    const int64_t* __restrict__ draft_ids, int K, int C, float temperature, int top_k, float top_p, uint64_t seed,
    const int64_t* __restrict__ verify_ids, const int64_t* __restrict__ eos, int n_eos,
    const int32_t* __restrict__ max_len, int32_t* __restrict__ start, int64_t* __restrict__ anchor,
    uint8_t* __restrict__ done, int64_t* __restrict__ out_tokens, int32_t* __restrict__ out_len, int64_t out_cap,
    int32_t* __restrict__ accepted_log, int32_t* __restrict__ cycle, int64_t log_cap) {
  __shared__ float sp[kSampleMaxBlock][kSampleMaxCand];
  __shared__ int first_reject;
  const int64_t b = blockIdx.x;
  const int i = threadIdx.x;
  if (done[b]) return;  // the same for the whole block
  const int block_len = min(K, max_len[b] - start[b]);
  const uint32_t cyc = static_cast<uint32_t>(cycle[b]);
  if (i == 0) first_reject = block_len - 1;
  if (i < K) sample_filter_row(vals + (b * K + i) * C, C, temperature, top_k, top_p, sp[i]);
  __syncthreads();
  if (i < block_len - 1) {
    const int64_t d = verify_ids[b * K + 1 + i];
    const int64_t qrow = b * (K - 1) + i;
    const float p = cand_prob(ids + (b * K + i) * C, sp[i], C, d);
    const float q = cand_prob(draft_ids + qrow * C, draft_probs + qrow * C, C, d);
    const float ratio = p / fmaxf(q, 1e-8f);
    const float u = sample_uniform(seed, static_cast<uint32_t>(b), cyc, static_cast<uint32_t>(i), kDrawAccept);
    if (!(u < fminf(ratio, 1.f))) atomicMin(&first_reject, i);
  }
  __syncthreads();
  if (i != 0) return;
  int accepted = first_reject;
  for (int j = 0; j < accepted; ++j) {  // stop after an accepted EOS, as the greedy cycle does
    if (is_eos(verify_ids[b * K + 1 + j], eos, n_eos)) {
      accepted = j + 1;
      break;
    }
  }
  const float* p = sp[accepted];
  const int64_t* pids = ids + (b * K + accepted) * C;
  float w[kSampleMaxCand];
  float total = 0.f;
  if (accepted < block_len - 1) {
    const int64_t qrow = b * (K - 1) + accepted;
    for (int j = 0; j < C; ++j) {
      w[j] = fmaxf(p[j] - cand_prob(draft_ids + qrow * C, draft_probs + qrow * C, C, pids[j]), 0.f);
      total += w[j];
    }
  }
  if (!(total > 1e-5f)) {
    total = 0.f;
    for (int j = 0; j < C; ++j) {
      w[j] = p[j];
      total += w[j];
    }
  }
  const float u = sample_uniform(seed, static_cast<uint32_t>(b), cyc, static_cast<uint32_t>(accepted), kDrawBonus);
  const int64_t bonus = pids[sample_pick(w, C, total, u)];
  commit_cycle(b, K, accepted, bonus, verify_ids, eos, n_eos, max_len, start, anchor, done, out_tokens, out_len,
               out_cap, accepted_log, cycle, log_cap);
}

// Philox4x32-10 of n (counter[4], key[2]) words, out [n, 4]: the generator's known-answer check.
__global__ void philox_kernel(const uint32_t* __restrict__ ck, int64_t n, uint32_t* __restrict__ out) {
  const int64_t r = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (r >= n) return;
  const uint32_t* c = ck + r * 6;
  const Philox4 v = philox4x32_10(c[0], c[1], c[2], c[3], c[4], c[5]);
  out[r * 4 + 0] = v.x;
  out[r * 4 + 1] = v.y;
  out[r * 4 + 2] = v.z;
  out[r * 4 + 3] = v.w;
}

}  // namespace orthrus
