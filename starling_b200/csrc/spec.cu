// The speculative verify / accept loop on the device (sb_spec_loop_*):
// SpeculativeDecoder.generate's loop (src/starling/granite/speculative.py:
// 400-539) as one CUDA graph,
//
//   setup kernel -> WHILE (continue) {
//                     SWITCH (k - 1) { verify forward of k + 1 tokens }
//                     control kernel
//                   }
//
// The verify forwards are the library's own sb_decode_step launches
// (VERIFY mode: per-row argmax into out_ids) captured once per chunk length.
// The control kernel applies the reference's rules to the argmaxes and
// writes the next round's ids and cache slot, then sets the SWITCH value
// (next k) and the WHILE condition.  It runs on every iteration, outside the
// SWITCH, and ends the loop after spec[SB_SPEC_MAX_ROUNDS] rounds whatever
// the state says, so the loop always terminates.  Both conditions reset to 0
// at every launch: the loop runs only once the setup kernel has turned it on.
#include <cstring>
#include <vector>

#include "common.cuh"

namespace sb {

namespace {

constexpr int kMinChunk = 8;       // speculative.py:295-303
constexpr int kBoundaryChunk = 2;
constexpr int kSearchWin = 40;     // re-alignment window (speculative.py:481-490)
constexpr int kStuckLimit = 8;     // stuck guard (speculative.py:492-497)
constexpr int kSpecThreads = 64;
constexpr int kMaxChunk = 16;                 // MAX_CHUNK (speculative.py:295-303)
constexpr int SB_MAX_VERIFY_ROWS = kMaxChunk + 1;

struct SpecArgs {
  int32_t* spec;
  int64_t* emitted;
  const int64_t* draft;
  int64_t* ids;       // shared ids of every verify state: [last, chunk...]
  int32_t* ctrl;      // shared ctrl block (SB_CTRL_SLOT = first slot of the verify)
  const int64_t* preds;  // shared out_ids: argmax of every verify row
  int64_t eos;
  int32_t max_chunk, max_len, emit_cap, draft_cap;
  cudaGraphConditionalHandle h_while, h_switch;
};

// Plan the next round (thread 0): k = min(chunk, n - draft_pos,
// max_new - n_emit, max_len - cache_pos - 1) (speculative.py:404-409); write
// [last emitted, draft[draft_pos : draft_pos + k]] and the cache slot, set
// the SWITCH to k - 1 and the WHILE to 1, or end the loop.
__device__ void plan_round(const SpecArgs& a) {
  int32_t* s = a.spec;
  const int n_draft = s[SB_SPEC_N_DRAFT], max_new = s[SB_SPEC_MAX_NEW];
  const int n_emit = s[SB_SPEC_N_EMIT], dp = s[SB_SPEC_DRAFT_POS], cp = s[SB_SPEC_CACHE_POS];
  int k = s[SB_SPEC_CHUNK];
  k = min(k, n_draft - dp);
  k = min(k, max_new - n_emit);
  k = min(k, a.max_len - cp - 1);
  const bool go = dp < n_draft && n_emit < max_new && k > 0 && k <= a.max_chunk && !s[SB_SPEC_STOPPED] &&
                  s[SB_SPEC_ROUNDS] < s[SB_SPEC_MAX_ROUNDS];
  if (!go) {
    if (dp < n_draft && n_emit < max_new && k > 0 && !s[SB_SPEC_STOPPED]) s[SB_SPEC_ERR] = 1;  // round limit
    s[SB_SPEC_K] = 0;
    cudaGraphSetConditional(a.h_switch, 0u);
    cudaGraphSetConditional(a.h_while, 0u);
    return;
  }
  a.ids[0] = a.emitted[n_emit - 1];
  for (int j = 0; j < k; ++j) a.ids[1 + j] = a.draft[dp + j];
  a.ctrl[SB_CTRL_SLOT] = cp;
  a.ctrl[SB_CTRL_PADLEN] = cp;
  s[SB_SPEC_K] = k;
  __threadfence();
  cudaGraphSetConditional(a.h_switch, static_cast<unsigned>(k - 1));
  cudaGraphSetConditional(a.h_while, 1u);
}

}  // namespace

// First node: state from the inputs the host wrote (N_DRAFT, MAX_NEW,
// PROMPT, MAX_ROUNDS; emitted[0] = the prefill's token), then the first round.
__global__ void k_spec_setup(const __grid_constant__ SpecArgs a) {
  if (threadIdx.x != 0) return;
  int32_t* s = a.spec;
  s[SB_SPEC_N_EMIT] = 1;
  s[SB_SPEC_CACHE_POS] = s[SB_SPEC_PROMPT];
  s[SB_SPEC_DRAFT_POS] = 0;
  s[SB_SPEC_CHUNK] = kMinChunk;
  s[SB_SPEC_STUCK] = 0;
  s[SB_SPEC_ACCEPTED] = 0;
  s[SB_SPEC_VERIFIES] = 0;
  s[SB_SPEC_ROUNDS] = 0;
  s[SB_SPEC_ERR] = 0;
  // the prefill token is EOS, or one token is all that was asked for (speculative.py:384-386)
  s[SB_SPEC_STOPPED] = a.emitted[0] == a.eos ? 1 : 0;
  plan_round(a);
}

// After each verify forward: the reference's accept / correct / bonus,
// cache rewind, re-alignment, stuck guard and chunk sizing
// (speculative.py:430-532), then the next round.
__global__ void __launch_bounds__(kSpecThreads) k_spec_control(const __grid_constant__ SpecArgs a) {
  __shared__ int64_t s_pred[SB_MAX_VERIFY_ROWS];
  __shared__ int64_t s_draft[SB_MAX_VERIFY_ROWS + kSearchWin];
  int32_t* s = a.spec;
  const int k = s[SB_SPEC_K];
  const int n_draft = s[SB_SPEC_N_DRAFT];
  const int dp0 = s[SB_SPEC_DRAFT_POS];
  // stage the argmaxes and the draft window this round can read
  for (int i = threadIdx.x; i <= k && i < SB_MAX_VERIFY_ROWS; i += blockDim.x) s_pred[i] = a.preds[i];
  for (int i = threadIdx.x; i < SB_MAX_VERIFY_ROWS + kSearchWin; i += blockDim.x)
    s_draft[i] = dp0 + i < n_draft ? a.draft[dp0 + i] : -1;
  __syncthreads();
  if (threadIdx.x != 0) return;
  s[SB_SPEC_ROUNDS] += 1;
  if (k < 1 || k > a.max_chunk) {  // no round was in flight: never loop on it
    s[SB_SPEC_ERR] = 1;
    cudaGraphSetConditional(a.h_while, 0u);
    return;
  }
  s[SB_SPEC_VERIFIES] += 1;
  int n_emit = s[SB_SPEC_N_EMIT];
  int dp = dp0, cp = s[SB_SPEC_CACHE_POS], accepted = s[SB_SPEC_ACCEPTED];
  auto emit = [&](int64_t t) {
    if (n_emit < a.emit_cap) a.emitted[n_emit] = t;
    ++n_emit;
  };
  int j = 0;
  bool mismatch = false, full = false, stopped = false;
  while (j < k && s_pred[j] == s_draft[j]) {  // accepted prefix
    emit(s_draft[j]);
    ++accepted;
    if (s_draft[j] == a.eos) {
      ++j;
      stopped = true;
      break;
    }
    ++j;
  }
  if (!stopped) {
    if (j < k) {  // the greedy correction
      emit(s_pred[j]);
      mismatch = true;
      stopped = s_pred[j] == a.eos;
    } else {  // everything accepted: the free bonus token
      full = true;
      emit(s_pred[k]);
      stopped = s_pred[k] == a.eos;
    }
  }
  if (full) {
    cp += k + 1;
    dp += k;
  } else if (mismatch) {
    cp += j + 1;
    dp += j;
  } else {
    cp += j;
    dp += j;
  }
  // re-align the draft on the last emitted token
  const int64_t last = a.emitted[min(n_emit, a.emit_cap) - 1];
  bool realigned = false;
  if (!stopped && dp < n_draft) {
    const int end = min(dp + kSearchWin, n_draft);
    for (int dd = dp; dd < end; ++dd) {
      if (s_draft[dd - dp0] == last) {
        dp = dd + 1;
        ++accepted;
        realigned = true;
        break;
      }
    }
  }
  int stuck = dp > dp0 ? 0 : s[SB_SPEC_STUCK] + 1;
  if (stuck >= kStuckLimit && !stopped && dp < n_draft) {
    dp = dp0 + 1;
    stuck = 0;
  }
  int chunk = s[SB_SPEC_CHUNK];
  if (!stopped) {
    if (full) chunk = min(chunk + 4, a.max_chunk);
    else if (mismatch && j == 0 && !realigned) chunk = kBoundaryChunk;
    else chunk = kMinChunk;
  }
  if (n_emit > a.emit_cap) s[SB_SPEC_ERR] = 1;
  s[SB_SPEC_N_EMIT] = min(n_emit, a.emit_cap);
  s[SB_SPEC_CACHE_POS] = cp;
  s[SB_SPEC_DRAFT_POS] = dp;
  s[SB_SPEC_ACCEPTED] = accepted;
  s[SB_SPEC_STUCK] = stuck;
  s[SB_SPEC_CHUNK] = chunk;
  s[SB_SPEC_STOPPED] = stopped ? 1 : 0;
  plan_round(a);
}

// ---- host side ------------------------------------------------------------------
struct SpecLoopGraph {
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
};

static int add_kernel(cudaGraphNode_t* node, cudaGraph_t g, const cudaGraphNode_t* deps, size_t ndeps,
                      void* func, const SpecArgs* args) {
  cudaKernelNodeParams kp;
  memset(&kp, 0, sizeof(kp));
  kp.func = func;
  kp.gridDim = dim3(1);
  kp.blockDim = dim3(kSpecThreads);
  void* argv[1] = {const_cast<SpecArgs*>(args)};
  kp.kernelParams = argv;
  note_launch();
  return cudaGraphAddKernelNode(node, g, deps, ndeps, &kp);
}

}  // namespace sb

using namespace sb;

extern "C" int sb_spec_loop_create(const SbModel* md, const SbSpecLoop* lp, void** out) {
  if (!md || !lp || !out || !lp->verify || !lp->spec || !lp->emitted || !lp->draft)
    return set_error(SB_ERR_ARG, "sb_spec_loop_create: null argument");
  if (lp->max_chunk < 1 || lp->max_chunk > kMaxChunk)
    return set_error(SB_ERR_ARG, "sb_spec_loop_create: max_chunk %d outside [1, %d]", lp->max_chunk, kMaxChunk);
  if (lp->emit_capacity < 2 || lp->draft_capacity < 1)
    return set_error(SB_ERR_ARG, "sb_spec_loop_create: capacities %d / %d", lp->emit_capacity, lp->draft_capacity);
  const SbState& v0 = lp->verify[0];
  for (int c = 0; c < lp->max_chunk; ++c) {
    const SbState& v = lp->verify[c];
    if (v.batch != 1 || v.m != c + 2 || v.mode != SB_MODE_VERIFY || v.ids != v0.ids || v.ctrl != v0.ctrl ||
        v.out_ids != v0.out_ids)
      return set_error(SB_ERR_ARG,
                       "sb_spec_loop_create: verify[%d] must be batch 1, m %d, VERIFY mode, sharing ids / ctrl / "
                       "out_ids with verify[0]", c, c + 2);
  }
  *out = nullptr;
  SpecLoopGraph* L = new SpecLoopGraph();
  cudaStream_t cs = nullptr;
  int rc = 0;
  auto cuda = [&](cudaError_t e, const char* what) {
    if (e != cudaSuccess && rc == 0) rc = set_error(e, "sb_spec_loop_create: %s: %s", what, cudaGetErrorString(e));
    return rc == 0;
  };
  SpecArgs a;
  memset(&a, 0, sizeof(a));
  a.spec = lp->spec;
  a.emitted = lp->emitted;
  a.draft = lp->draft;
  a.ids = v0.ids;
  a.ctrl = v0.ctrl;
  a.preds = v0.out_ids;
  a.eos = lp->eos_id;
  a.max_chunk = lp->max_chunk;
  a.max_len = md->max_len;
  a.emit_cap = lp->emit_capacity;
  a.draft_cap = lp->draft_capacity;
  cudaGraphNode_t while_node = nullptr, switch_node = nullptr, setup_node = nullptr, ctl_node = nullptr;
  cudaGraph_t body = nullptr;
  std::vector<cudaGraph_t> cases;
  if (cuda(cudaGraphCreate(&L->graph, 0), "cudaGraphCreate") &&
      cuda(cudaGraphConditionalHandleCreate(&a.h_while, L->graph, 0, cudaGraphCondAssignDefault), "while handle")) {
    cudaGraphNodeParams np = {cudaGraphNodeTypeConditional};
    np.conditional.handle = a.h_while;
    np.conditional.type = cudaGraphCondTypeWhile;
    np.conditional.size = 1;
    if (cuda(cudaGraphAddNode(&while_node, L->graph, nullptr, 0, &np), "while node")) body = np.conditional.phGraph_out[0];
  }
  if (rc == 0 && cuda(cudaGraphConditionalHandleCreate(&a.h_switch, body, 0, cudaGraphCondAssignDefault), "switch handle")) {
    cudaGraphNodeParams np = {cudaGraphNodeTypeConditional};
    np.conditional.handle = a.h_switch;
    np.conditional.type = cudaGraphCondTypeSwitch;
    np.conditional.size = static_cast<unsigned>(lp->max_chunk);
    if (cuda(cudaGraphAddNode(&switch_node, body, nullptr, 0, &np), "switch node"))
      cases.assign(np.conditional.phGraph_out, np.conditional.phGraph_out + lp->max_chunk);
  }
  // case c: the verify forward of c + 2 tokens, captured from the library's own launches
  if (rc == 0 && cuda(cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking), "stream")) {
    for (int c = 0; c < lp->max_chunk && rc == 0; ++c) {
      if (!cuda(cudaStreamBeginCaptureToGraph(cs, cases[c], nullptr, nullptr, 0, cudaStreamCaptureModeThreadLocal),
                "begin capture"))
        break;
      const int r = sb_decode_step(md, &lp->verify[c], 0, cs);
      cudaGraph_t got = nullptr;
      const cudaError_t e = cudaStreamEndCapture(cs, &got);
      if (r != 0 && rc == 0) rc = r;  // message already set by sb_decode_step
      cuda(e, "end capture");
    }
  }
  if (rc == 0) cuda(static_cast<cudaError_t>(add_kernel(&ctl_node, body, &switch_node, 1,
                                                        reinterpret_cast<void*>(k_spec_control), &a)),
                    "control node");
  if (rc == 0) cuda(static_cast<cudaError_t>(add_kernel(&setup_node, L->graph, nullptr, 0,
                                                        reinterpret_cast<void*>(k_spec_setup), &a)),
                    "setup node");
  if (rc == 0) cuda(cudaGraphAddDependencies(L->graph, &setup_node, &while_node, 1), "setup -> while");
  if (rc == 0) cuda(cudaGraphInstantiate(&L->exec, L->graph, 0), "instantiate");
  if (cs) cudaStreamDestroy(cs);
  if (rc != 0) {
    sb_spec_loop_destroy(L);
    return rc;
  }
  *out = L;
  return 0;
}

extern "C" int sb_spec_loop_launch(void* loop, sb_stream_t stream) {
  SpecLoopGraph* L = static_cast<SpecLoopGraph*>(loop);
  if (!L || !L->exec) return set_error(SB_ERR_ARG, "sb_spec_loop_launch: no loop");
  const cudaError_t e = cudaGraphLaunch(L->exec, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return set_error(e, "sb_spec_loop_launch: %s", cudaGetErrorString(e));
  return 0;
}

extern "C" void sb_spec_loop_destroy(void* loop) {
  SpecLoopGraph* L = static_cast<SpecLoopGraph*>(loop);
  if (!L) return;
  if (L->exec) cudaGraphExecDestroy(L->exec);
  if (L->graph) cudaGraphDestroy(L->graph);
  delete L;
}
