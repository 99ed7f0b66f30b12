// Launch descriptors shared by the host dispatch code and the AFA kernels.
//
// A launch covers up to kMaxProblems "problems". A problem is one contiguous
// block of query rows (a q segment) attending to one or two key segments. Each
// segment carries the global sequence position of its first row, so causal
// visibility (key_pos <= query_pos, src/kernels/pallas_afa.py:121-124 and the
// global-position form of the ring at :640-646) is decided on global positions
// and one kernel serves the single-device forward, every ring hop and decode.
#pragma once

#include <cstdint>

namespace afa {

constexpr int kMaxProblems = 4;
constexpr int kMaxKSegs = 2;

struct Segment {
  int row0;  // first row of the segment in the per-(batch,head) tensor
  int len;   // number of rows (keys beyond len are masked, like valid_seq_len)
  int pos0;  // global sequence position of row0
};

struct Problem {
  Segment q;
  Segment k[kMaxKSegs];
  int nk;       // number of key segments (1 or 2)
  int cta0;     // first CTA (along the problem axis of the grid) of this problem
  int ncta;     // CTAs of this problem
};

enum EpilogueMode : int {
  kFinal = 0,       // out = O / (d + sink) in the input dtype; d_total = d + sink
  kStoreRaw = 1,    // o_acc = O, d_acc = d (fp32 / fp64 accumulators)
  kAccumRaw = 2,    // o_acc += O, d_acc += d
  kAccumFinal = 3,  // out = (o_acc + O) / (d_acc + d + sink); d_total = d_acc + d + sink
};

struct Launch {
  Problem prob[kMaxProblems];
  int nprob;
  int causal;
  int mode;
  int B, H;
  int lq;   // rows per (batch, head) of Q and of out / o_acc
  int lk;   // rows per (batch, head) of K and V
  int d;    // head dimension
  float scale;
  float sink;
  double scale_d;
  double sink_d;
  const void* q;
  const void* k;
  const void* v;
  void* out;      // kFinal / kAccumFinal: output in the input dtype
  void* dtot;     // kFinal / kAccumFinal: denominator (accumulation dtype), may be null
  void* o_acc;    // raw modes: numerator accumulator (accumulation dtype)
  void* d_acc;    // raw modes: row-sum accumulator (accumulation dtype)
  int* status;    // device status word (0 = ok)
};

// Device status codes written by kernels (bounded waits that ran out).
enum DeviceStatus : int {
  kDevOk = 0,
  kDevTimeoutProducer = 0x101,
  kDevTimeoutMma = 0x102,
  kDevTimeoutSoftmax = 0x103,
  kDevTimeoutEpilogue = 0x104,
  kDevTimeoutDrain = 0x105,
  kDevTimeoutSelftest = 0x1ff,
};

}  // namespace afa
