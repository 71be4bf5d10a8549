// Split-K merge for the decode kernels: last-arriver, no extra launch.
//
// Every split CTA of one (sequence, kv head) stores its softmax state
// (m, l in the log2 domain, unnormalised acc[D] per query head) in the
// workspace, then arrives on that pair's counter.  The CTA that arrives last
// reads all states back, writes the normalised output and puts the counter
// back to zero, so the counter words stay zero between launches: a caller
// zero-fills the workspace once and may reuse it for every later launch that
// is not concurrent with another one using it.  The counters sit in a
// fixed-size region at the start of the workspace, so the states of a launch
// of any shape never land on a counter word of a later launch.  No CTA ever
// waits for another (the merge is done by whichever CTA finishes last), so
// the scheme needs no co-scheduling and no cluster.
//
// Workspace layout (mi_paged_decode_workspace_bytes):
//   int32 counters[kSplitCounters]            (64 KiB, whatever the shape)
//   f32   acc[num_seqs * num_q_heads * splits][head_dim]
//   f32   ml[num_seqs * num_q_heads * splits][2]
// State index (seq * num_q_heads + q head) * splits + split; counter index
// seq * num_kv_heads + kv head (< kSplitCounters).
#pragma once

#include "common.cuh"
#include "params.cuh"

namespace mi {

constexpr int64_t kSplitCounters = 16384;  // (seq, kv head) pairs one split launch can hold
constexpr size_t kSplitCounterBytes = kSplitCounters * sizeof(int32_t);

// Point the decode parameters at a workspace laid out as above.
inline void set_split_workspace(DecodeParams &p, void *workspace, int64_t num_seqs,
                                int32_t num_q_heads, int32_t head_dim, int nsplit) {
  const size_t states = static_cast<size_t>(num_seqs) * num_q_heads * nsplit;
  char *base = static_cast<char *>(workspace);
  p.ws_count = reinterpret_cast<int32_t *>(base);
  p.ws_acc = reinterpret_cast<float *>(base + kSplitCounterBytes);
  p.ws_ml = p.ws_acc + states * head_dim;
}

// Store this split's state for head h, element d (thread-parallel over (h, d)).
__device__ __forceinline__ void split_store_state(const DecodeParams &p, int64_t seq, int qh,
                                                  int nsplit, int split, int D, int d, float M,
                                                  float L, float A) {
  const int64_t state = (seq * p.num_q_heads + qh) * nsplit + split;
  p.ws_acc[state * D + d] = A;
  if (d == 0) {
    p.ws_ml[state * 2] = M;
    p.ws_ml[state * 2 + 1] = L;
  }
}

// Called by every thread of the CTA after its states are stored: arrive on the
// counter and, in the last CTA, merge all splits into `out`.
template <typename T, int G, int D>
__device__ __forceinline__ void split_arrive_and_merge(const DecodeParams &p, int64_t seq, int kvh,
                                                       int nsplit, int *last_smem) {
  __threadfence();  // this thread's state stores are visible GPU-wide before the arrival
  __syncthreads();
  int *counter = p.ws_count + seq * p.num_kv_heads + kvh;
  if (threadIdx.x == 0) {
    const int before = atomicAdd(counter, 1);
    *last_smem = before == nsplit - 1;
    __threadfence();
  }
  __syncthreads();
  if (!*last_smem) return;
  __threadfence();
  for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
    const int h = i / D, d = i % D;
    const int qh = kvh * G + h;
    const int64_t s0 = (seq * p.num_q_heads + qh) * nsplit;
    float M = -INFINITY;
    for (int s = 0; s < nsplit; ++s) M = fmaxf(M, __ldcg(p.ws_ml + (s0 + s) * 2));
    float L = 0.f, A = 0.f;
#pragma unroll 4
    for (int s = 0; s < nsplit; ++s) {
      const float ms = __ldcg(p.ws_ml + (s0 + s) * 2);
      const float ls = __ldcg(p.ws_ml + (s0 + s) * 2 + 1);
      const float as = __ldcg(p.ws_acc + (s0 + s) * D + d);
      if (ms != -INFINITY) {
        const float f = fast_exp2(ms - M);
        L += f * ls;
        A += f * as;
      }
    }
    T *o = static_cast<T *>(p.out) + (seq * p.num_q_heads + qh) * D;
    o[d] = Elem<T>::from_float(L > 0.f ? A / L : 0.f);
  }
  if (threadIdx.x == 0) *counter = 0;  // every split has arrived: ready for the next launch
}

}  // namespace mi
