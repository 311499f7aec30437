// sg_gemv.cu -- decode GEMV (batch 1..16) for Q4_0 / Q4_K on B200 tensor
// cores (tcgen05 kind::i8, operands and accumulators in TMEM).
//
// Replaces the engine's per-token GEMV routes: forward_linear's Q4_0 path
// (swamp-engine/src/linear.rs:68-87: dequant + f32 row dots) and
// fused_gemv_q4k (swamp-kernels/src/fused_gemv_q4k.rs:59-82, scalar order
// :466-508), plus forward_linear_multi (linear.rs:96-170) when several
// tensors share one x.
//
// Arithmetic. Per 32-element block b of row r (Q4_0: w = d*(q-8); Q4_K:
// w = sv*q - mv with sv = d*sc, mv = dmin*m):
//   y[t][r] = sum_b ( sv_b * sum_{k in b} q_k x_k  -  mv_b * sum_{k in b} x_k )
// The integer part runs on the tensor core, exactly: A holds the raw nibbles
// q as u8, B holds the activations as three signed 8-bit digits. Per unit of
// 256 K and token, x is scaled by a power of two s (max |x| * s in [32, 64))
// and rounded to V = rint(x * s * 2^14), |V| <= 2^20, which splits exactly
// into V = d0 * 2^14 + d1 * 2^7 + d2 with every digit in [-64, 64].
// D_i = sum_k q_k d_i,k per 32-block is exact in s32 (|D_i| < 2^15); the
// epilogue rebuilds sum q u = D0 + D1/128 + D2/16384 (u = V / 2^14) exactly
// before one rounding, subtracts the block's constant part (sum u, computed
// from the same digits) and applies the block scales in f32; per unit the
// sum is scaled back by 1/s.
//
// Block-diagonal activation tiles. One MMA covers one 32-block (K = 32
// bytes), and every block needs its own columns (its scales differ per
// row). Instead of one accumulator per block, each chunk's activation tile
// gives every (block, digit, token) its own row of B, holding that block's
// digits in the block's half of K and zeros elsewhere; all MMAs of GC chunks
// then accumulate into one accumulator of N = GC*6*BT columns (padded to
// 16), each block landing in its own columns. At one token a whole 256-K
// unit needs 32 TMEM columns instead of 8 x 16, so several groups fit in
// flight.
//
// Work split: the chunks (128 rows x 64 K, one 4608-byte tile each) of all
// row-blocks of all matrices form one sequence, row-block major; CTA c of G
// takes chunks [c*T/G, (c+1)*T/G). It walks them in pieces -- the part of
// one unit (4 consecutive chunks = 256 K = one Q4_K super-block) inside its
// range -- so each piece's weights arrive in one bulk copy (bandwidth comes
// from large copies). A row-block covered by one CTA is stored directly;
// one shared by several CTAs is reduced into y with red.add: the CTA holding
// its first chunks zeroes its rows when the kernel starts and publishes the
// call's epoch in a flag of the workspace after its first group; the other
// CTAs confirm the flag (read early, checked at the end of their segment)
// before their first red.add. With SG_FLAG_ACCUMULATE nothing is zeroed.
//
// One kernel per call (plus gemv_xprep_kernel from 4 tokens on). Roles, all
// decoupled by mbarrier rings (the exact warp map and ring depths per batch
// are in Cfg):
//   weights     warp 0 lane 0: one cp.async.bulk per piece into a ring of
//               weight slots, issued from CTA entry (weights do not depend on
//               the previous kernel); spare lanes zero shared output rows.
//   dequant     warps 2-5, one weight row per thread: two 16-byte reads and
//               eight masks per 32-block, one tcgen05.st of the chunk's 64 u8
//               into the row's TMEM lane, and the group's scale words.
//   MMA         one thread per issuer: tcgen05.mma kind::i8 (M=128, K=32, A
//               from TMEM, B = activation tile in shared memory), commits to
//               the accumulator slot and to the A-tile slot.
//   epilogue    4 warps per set (warp % 4 = TMEM lane quadrant): tcgen05.ld of
//               the accumulators and scale words, block scales in f32, rows
//               stored or reduced at segment ends.
//   activations 1-2 tokens: warps convert x to digit tiles per piece; from 4
//               tokens: one thread bulk-copies the prepared unit images.
// One thread issues an MMA about every 50 cycles and every role's loop costs
// about as much per piece as HBM takes to deliver it to one SM, so the
// configurations multiply independent pipelines: two CTAs per SM at one
// token, two MMA issuers and two epilogue sets taking alternate pieces at 2
// and 4 tokens. TMEM holds two rings: A-tile slots (free once the MMAs that
// read them complete) and accumulator slots with the scale words (free once
// the epilogue read them). Every mbarrier wait is bounded (sg_common.cuh).
#include <algorithm>
#include <atomic>
#include <climits>

#include "sg_gemv.cuh"
#include "sg_tc.cuh"

namespace gemv_tc {

constexpr int kUC = 4;                          // chunks per unit
constexpr int kACols = 16;                      // TMEM columns of one chunk's A tile: 64 K of u8 per lane
constexpr int kScCols = 5;                      // TMEM columns of a group's scale words (chunks 0..3, Q4_K d|dmin at 4)
constexpr int kWU = kUC * SG_TILE_BYTES + 512;  // packed weights of a unit + Q4_K d|dmin
constexpr int kMaxCtas = SG_GEMV_MAX_CTAS;
constexpr int kSumOff = 0;                      // within a unit's tail: block sums [chunk 4][blk 2][token 16] f32
constexpr int kInvOff = 512;                    //                       1/s per token [16] f32

template <int BT>
struct Cfg {
  // Every role's loop has a fixed cost per piece (waits, hand-offs) of the
  // order of the time HBM takes to deliver the piece to one SM. At one token
  // two CTAs share each SM (CPS), each with half the rings: two independent
  // pipelines per SM. Wider batches need the registers of a whole SM.
  static constexpr bool DUAL = BT == 1;
  static constexpr int CPS = DUAL ? 2 : 1;                   // CTAs per SM
  static constexpr int GC = BT <= 2 ? 4 : BT == 16 ? 1 : 2;   // chunks per accumulator
  // From 4 tokens on, the activation tiles are built once per call by
  // gemv_xprep_kernel (an image in global memory, one bulk copy per piece):
  // converting them in every CTA would repeat the work for each row-block.
  // Work is then split on GC-chunk boundaries, so a chunk's accumulator
  // position is always chunk % GC.
  static constexpr bool XPRE = BT >= 4;
  static constexpr int SPL = XPRE ? GC : 1;                  // work split granularity (chunks)
  static constexpr int CPG = BT >= 8 ? 2 : 4;                // chunks per group (one hand-off between roles)
  static constexpr int NACC = CPG / GC;                      // accumulators per group
  static constexpr int ROWS = GC * 6 * BT;                   // B rows: (chunk, block, digit, token)
  static constexpr int N = (ROWS + 15) / 16 * 16;            // MMA N
  static constexpr int T = N * 64;                           // activation tile bytes (one chunk)
  static constexpr int XU = kUC * T + 1024;                  // activation unit: 4 tiles + sums + scales
  // activation unit ring: a slot is held from its conversion or copy until
  // the epilogue has read the unit's sums, a loop of several microseconds
  static constexpr int RX = DUAL ? 4 : BT <= 4 ? 6 : 4;
  // Activations built in the kernel (1 or 2 tokens): NXW warps, XPP of them
  // (one per token) on each piece, the pieces dealt round-robin to XL =
  // NXW / XPP lanes of warps. Converting a unit is a chain of shuffles of
  // about 0.8 us per warp, so several pieces must be in conversion at once.
  static constexpr int NXW = XPRE ? 1 : DUAL ? 2 : 4;        // activation warps (with XPRE: the copy thread's)
  static constexpr int XPP = XPRE ? 1 : BT;                  // warps (tokens) per piece
  static constexpr int XL = NXW / XPP;                       // pieces converted side by side
  static constexpr int XS = XPRE ? 0 : 3;                    // staging slots per activation warp (x prefetch)
  // One thread issues an MMA about every 50 cycles whatever its size, and
  // issuers in different warps run side by side; a group's epilogue is a
  // chain of waits and loads of similar latency. Up to 4 tokens a group is
  // one piece, and two lanes -- an MMA issuer and a set of 4 epilogue warps
  // each -- take alternate pieces: set s the pieces v with v % 2 == s.
  static constexpr int NSET = !DUAL && BT <= 4 ? 2 : 1;
  // Warps: 0 weights (lane 0) and shared output rows; 1 MMA issuer 0 and
  // TMEM owner; 2-5 dequant; 6-9 epilogue set 0; 10 (and 11, 17, 18 when
  // x is converted here) activations; 12-15 epilogue set 1; MMA issuer 1 at
  // 16 (11 when x is prepared).
  static constexpr int WARPS = DUAL ? 12 : BT == 2 ? 19 : BT == 4 ? 16 : 12;
  static constexpr int THREADS = WARPS * 32;
  // Registers per thread: a GEMV CTA leaves room for one CTA of the next
  // call's activation prep kernel (128 threads x 32 registers), which under
  // programmatic dependent launch must run on an SM next to it; at one token
  // two GEMV CTAs share the SM.
  static constexpr int MAXREG = DUAL ? 80 : ((65536 - 4096) / THREADS) / 8 * 8;
  static constexpr int MMA1_WARP = BT <= 2 ? 16 : 11;
  // activation warp index of `warp` (-1: not one)
  __device__ static int x_warp(int warp) {
    if (warp == 10) return 0;
    if (!XPRE && warp == 11) return 1;
    if (!XPRE && !DUAL && (warp == 17 || warp == 18)) return warp - 15;
    return -1;
  }
  static constexpr int OFF_X = 0;
  static constexpr int OFF_S = OFF_X + RX * XU;              // x staging: [warp][slot][256] f32
  static constexpr int OFF_W = OFF_S + NXW * XS * 1024;
  // One CTA per SM: two CTAs of consecutive calls sharing an SM under PDL
  // would make the second wait in tcgen05.alloc; ask for more than half of
  // the SM's shared memory.
  // Weight ring: a slot holds a piece from its copy until the dequant warps
  // have read it; at one CTA per SM the copies in flight must cover the HBM
  // latency under load (about 2 us at 44 GB/s per SM), so the ring takes
  // what shared memory leaves.
  static constexpr int RW = DUAL ? 3 : BT <= 4 ? 7 : 6;
  static constexpr int SMEM_USED = OFF_W + RW * kWU + 1024;
  static constexpr int SMEM = DUAL || SMEM_USED > 120 * 1024 ? SMEM_USED : 120 * 1024;
  // TMEM holds two rings. A-tile slots (SA) are free again once the MMAs
  // that read them complete; accumulator slots (SD, each with the group's
  // scale words) once the epilogue has read them. The dequant warps thus
  // wait on the short dequant -> MMA loop for A, and the long loop through
  // the epilogue is covered by the deeper accumulator ring. Layout:
  // [SD accumulator blocks][SA A-tile blocks][SD x kScCols scale words];
  // every multi-column access starts on a multiple of 16 columns, scale
  // words are read and written one column at a time.
  static constexpr uint32_t A_COLS = CPG * kACols;
  static constexpr uint32_t D_COLS = NACC * N;
  static constexpr uint32_t TMEM_COLS = DUAL ? 256 : 512;
  static constexpr int SA = DUAL ? 2 : 3;
  static constexpr int SD_FIT = (int)((TMEM_COLS - SA * A_COLS) / (D_COLS + kScCols));
  static constexpr int SD = SD_FIT > 6 ? 6 : SD_FIT;
  static constexpr uint32_t A_COL0 = SD * D_COLS;
  static constexpr uint32_t SC_COL0 = A_COL0 + SA * A_COLS;
  __host__ __device__ static constexpr uint32_t d_col(int sd) { return (uint32_t)sd * D_COLS; }
  __host__ __device__ static constexpr uint32_t a_col(int sa) { return A_COL0 + (uint32_t)sa * A_COLS; }
  __host__ __device__ static constexpr uint32_t sc_col(int sd) { return SC_COL0 + (uint32_t)sd * kScCols; }
  static constexpr uint32_t IDESC = sg_idesc_u8s8(128, N);
  static_assert(SA >= 2 && SD >= 2 && SC_COL0 + SD * kScCols <= TMEM_COLS, "TMEM budget");
  static_assert(D_COLS % 16 == 0 && A_COLS % 16 == 0, "TMEM alignment");
  static_assert(N <= 256 && ROWS <= N, "MMA N");
  static_assert(XU % 1024 == 0, "operand tiles keep 1024-byte alignment");
  static_assert(SMEM_USED <= (DUAL ? 110 : 227) * 1024, "shared memory budget");
  static_assert(NSET == 1 || (CPG == kUC && BT <= 4), "two lanes need one group per piece");
  // epilogue TMEM loads: LC columns at a time, whole (position, block) column
  // groups of 3 x BT each (fewer live registers at 8 and 16 tokens)
  static constexpr int LC = N < 48 ? N : 48;
  static_assert(LC % 16 == 0 && (LC % (3 * BT) == 0 || 2 * GC * 3 * BT <= LC), "epilogue load split");
  static_assert(XPRE || (BT <= 2 && XL * XPP == NXW && RX % XL == 0), "activation lanes");
};

struct Mat {
  const uint8_t* tiles;
  const uint32_t* dd;
  float* y;
  int64_t ldy;
  int n_rb, n_rows, n_sb, rb0;
};

struct Params {
  Mat mats[SG_GEMV_MAX_MATS];
  int n_mats, batch, n_ch, accumulate;
  int n_cp;        // chunks per row-block in the work index, n_ch rounded up to the split granularity
  int spl;         // split granularity: CTA ranges start and end on multiples of it
  int64_t total;   // work-index chunks over all row-blocks of all matrices (n_cp per row-block)
  uint8_t* ximg;   // activation unit images (gemv_xprep_kernel), when the configuration uses them
  const float* x;  // [batch][ldx]
  int64_t ldx;
  int K;
  unsigned long long* zflags;  // [kMaxCtas][4]: epoch once CTA c zeroed the shared rows of lane quadrant q
  unsigned long long epoch;    // this call's epoch (never 0, never repeated)
};

__device__ __forceinline__ int find_mat(const Params& p, int rbg) {
  int m = 0;
#pragma unroll
  for (int i = 1; i < SG_GEMV_MAX_MATS; ++i)
    if (i < p.n_mats && rbg >= p.mats[i].rb0) m = i;
  return m;
}

// CTA whose chunk range holds global chunk gc (range of c: [c*T/G, (c+1)*T/G))
__device__ __forceinline__ int cta_of(const Params& p, int64_t gc) {
  const int64_t ts = p.total / p.spl;
  return (int)(((gc / p.spl + 1) * (int64_t)gridDim.x - 1) / ts);
}
// the work-index chunk range [g0, g1) of CTA b (multiples of spl)
__device__ __forceinline__ void cta_range(const Params& p, int b, int64_t& g0, int64_t& g1) {
  const int64_t ts = p.total / p.spl;
  g0 = (int64_t)b * ts / gridDim.x * p.spl;
  g1 = (int64_t)(b + 1) * ts / gridDim.x * p.spl;
}

// Piece cursor over the CTA's chunk range [g, g1).
struct Cursor {
  int rbg, c, mi, rb;  // global row-block, chunk within it, matrix, row-block within the matrix
  int g, g1;           // work index (the host keeps the total below 2^31)
  int nrb0;            // first global row-block of the next matrix
  __device__ __forceinline__ void init(const Params& p, int64_t g0, int64_t gend) {
    g = (int)g0;
    g1 = (int)gend;
    rbg = g / p.n_cp;
    c = g - rbg * p.n_cp;  // range ends never fall in the padding
    mi = find_mat(p, rbg);
    rb = rbg - p.mats[mi].rb0;
    nrb0 = mi + 1 < p.n_mats ? p.mats[mi + 1].rb0 : INT_MAX;
  }
  __device__ __forceinline__ bool more() const { return g < g1; }
  __device__ __forceinline__ int sc() const { return c >> 2; }
  __device__ __forceinline__ int ci0() const { return c & 3; }
  __device__ __forceinline__ int cnt(const Params& p) const { return min(min(kUC - (c & 3), p.n_ch - c), g1 - g); }
  __device__ __forceinline__ void next(const Params& p) {
    const int n = cnt(p);
    g += n;
    c += n;
    if (c == p.n_ch) {
      g += p.n_cp - p.n_ch;  // skip the padding of the work index
      c = 0;
      ++rbg;
      ++rb;
      if (rbg >= nrb0) {
        ++mi;
        rb = 0;
        nrb0 = mi + 1 < p.n_mats ? p.mats[mi + 1].rb0 : INT_MAX;
      }
    }
  }
};


// Position in a ring of R mbarrier-guarded slots: the slot and the parity
// of its current phase, stepped without division.
template <int R, int S = 1>
struct Ring {
  int slot;
  uint32_t phase;
  __device__ __forceinline__ explicit Ring(int start = 0) : slot(start), phase(0u) {}  // start < R
  __device__ __forceinline__ void next() {  // S positions on (S <= R)
    slot += S;
    if (slot >= R) {
      slot -= R;
      phase ^= 1u;
    }
  }
};

// 16-byte segment j of row r of a K-major SWIZZLE_64B tile (64-byte rows)
__device__ __forceinline__ int sw64_off(int r, int j) { return r * 64 + ((j ^ ((r >> 1) & 3)) << 4); }

// ------------------------------------------------------- activation digits
// For unit sc and token t, lane l of a warp holds K = 256 sc + 8l + e,
// e = 0..7: chunk l/8 of the unit, 32-block (l%8)/4 of the chunk, layout
// word l%4 of the block. The unit's max |x| sets s = 2^se with max*s in
// [32, 64); V = rint(x*s*2^14) = d0*2^14 + d1*2^7 + d2, every digit in
// [-64, 64]. Digit i of the lane's 8 values is packed as two 32-bit words
// whose bytes hold K offsets {0,4,1,5} and {2,6,3,7} -- the order in which a
// layout word's low and high nibbles come out of one mask each. Per unit the
// tail holds sums[chunk 4][blk 2][token 16] = sum_k V/2^14 over the 32-block
// and inv[16] = 1/s (NaN when the unit holds a non-finite x, so the output
// is non-finite too). K beyond the matrix reads as zero.
struct UnitDigits {
  uint32_t dig[3][2];
  int vsum;    // sum of the lane's V
  bool bad;    // the unit holds a non-finite x
  int se;
};

__device__ __forceinline__ void load_x8(const Params& p, int sc, int t, int lane, float (&v)[8]) {
  const int k0 = 256 * sc + 8 * lane;
  if (t < p.batch && k0 < p.K) {
    const float* xr = p.x + (int64_t)t * p.ldx + k0;
    const float4 a = *reinterpret_cast<const float4*>(xr);
    const float4 b = *reinterpret_cast<const float4*>(xr + 4);
    v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = 0.f;
  }
}

// warp-collective: every lane of the warp calls it for the same token
__device__ __forceinline__ UnitDigits unit_digits(const float (&v)[8]) {
  UnitDigits u;
  float m = 0.f;
  bool bad = false;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    m = fmaxf(m, fabsf(v[e]));
    bad |= !(fabsf(v[e]) <= 3.402823466e38f);  // inf or NaN
  }
  // m >= 0 and not NaN (fmaxf drops NaN), so its bits order like its value:
  // one warp reduction instead of a chain of shuffles
  m = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(m)));
  u.bad = __any_sync(0xffffffffu, bad);
  u.se = 0;  // s = 2^se, with 1/s a normal float as well
  if (m > 0.f && !u.bad) {
    const int e = ((__float_as_int(m) >> 23) & 0xFF) - 127;  // m in [2^e, 2^(e+1)) for normal m
    u.se = max(-126, min(126, 5 - e));
  }
  const float s = __int_as_float((127 + u.se) << 23);
  int V[8];
  u.vsum = 0;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    V[e] = u.bad ? 0 : __float2int_rn((v[e] * s) * 16384.f);
    u.vsum += V[e];
  }
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    uint32_t w0 = 0, w1 = 0, w2 = 0;
#pragma unroll
    for (int pb = 0; pb < 4; ++pb) {
      const int e = (pb & 1) * 4 + (pb >> 1) + 2 * half;  // byte pb of the low / high word: K 0,4,1,5 | 2,6,3,7
      const int d0 = (V[e] + 8192) >> 14;
      const int r0 = V[e] - (d0 << 14);
      const int d1 = (r0 + 64) >> 7;
      const int d2 = r0 - (d1 << 7);
      w0 |= (uint32_t)(d0 & 0xFF) << (8 * pb);
      w1 |= (uint32_t)(d1 & 0xFF) << (8 * pb);
      w2 |= (uint32_t)(d2 & 0xFF) << (8 * pb);
    }
    u.dig[0][half] = w0;
    u.dig[1][half] = w1;
    u.dig[2][half] = w2;
  }
  return u;
}

// the per-block sums and the token's 1/s into a unit's tail (warp-collective)
__device__ __forceinline__ void store_tail(float* tail, const UnitDigits& u, int t, int lane) {
  int vs = u.vsum;
  vs += __shfl_xor_sync(0xffffffffu, vs, 1);
  vs += __shfl_xor_sync(0xffffffffu, vs, 2);  // 4 lanes = one 32-block
  if ((lane & 3) == 0) tail[kSumOff / 4 + ((lane >> 3) * 2 + ((lane >> 2) & 1)) * 16 + t] = (float)vs * (1.f / 16384.f);
  if (lane == 0) tail[kInvOff / 4 + t] = u.bad ? __int_as_float(0x7fc00000) : __int_as_float((127 - u.se) << 23);
}

// B row of (position k of a chunk in its accumulator, block j, digit d,
// token t) in the chunk's tile. A piece's chunk i (i = chunk - first chunk
// of the piece) has position i % GC, so a position is a compile-time index
// in the epilogue.
template <int BT>
__host__ __device__ constexpr int brow(int k, int j, int d, int t) {
  return (k * 2 + j) * 3 * BT + d * BT + t;
}

// Block-diagonal tile of a chunk (K-major, 64-byte swizzle): row brow(k, j,
// d, t) holds the digits in bytes 32j .. 32j+31, zeros elsewhere (the slots
// are zeroed at kernel start and only digit bytes are written). Lanes of
// chunks before ci0 (outside the piece) write nothing.
template <int BT>
__device__ __forceinline__ void store_digits(uint8_t* unit, const UnitDigits& u, int t, int lane, int ci0) {
  using C = Cfg<BT>;
  const int c = lane >> 3, j = (lane >> 2) & 1, w = lane & 3;
  if (c >= ci0) {
    uint8_t* tile = unit + c * C::T;
#pragma unroll
    for (int d = 0; d < 3; ++d) {
      const int n = brow<BT>((c - ci0) % C::GC, j, d, t);
      *reinterpret_cast<uint2*>(tile + sw64_off(n, 2 * j + (w >> 1)) + 8 * (w & 1)) = make_uint2(u.dig[d][0], u.dig[d][1]);
    }
  }
  store_tail(reinterpret_cast<float*>(unit + kUC * C::T), u, t, lane);
}

// N consecutive TMEM columns of this warp's lane quadrant (N a multiple of 16)
template <int N>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t (&v)[N]) {
#pragma unroll
  for (int i = 0; i + 32 <= N; i += 32) sg_tmem_ld_n<32>(taddr + i, *reinterpret_cast<uint32_t(*)[32]>(&v[i]));
  if constexpr (N % 32 == 16) sg_tmem_ld_n<16>(taddr + (N - 16), *reinterpret_cast<uint32_t(*)[16]>(&v[N - 16]));
}

// sum_k q_k u_k = D0 + D1/128 + D2/16384, rounded once: D0*128 + D1
// (|.| < 2^22) and D2 become floats exactly by adding them to the bits of
// 1.5*2^23 and 1.5*2^9; the two 1.5 offsets cancel (-98304 - 768 + 768).
__device__ __forceinline__ float digit_dot(uint32_t d0, uint32_t d1, uint32_t d2) {
  const float f = __uint_as_float(d0 * 128u + d1 + 0x4B400000u);
  const float u = fmaf(f, 0.0078125f, -99072.f);
  const float g = __uint_as_float(d2 + 0x44400000u);
  return u + g;
}

// ----------------------------------------------------- output row-blocks
// A row-block segment (the rows a CTA accumulates between two stores) is
// stored when the CTA ran the whole row-block, else reduced into y with
// red.add. Before the first reduction into a shared row-block, its rows must
// have been zeroed by the CTA holding the row-block's first chunk. Spare
// lanes of warp 0 do that work off the critical path (shared_rows_role):
// they zero this CTA's trailing row-block and publish the call's epoch in
// the CTA's flag (then arrive on zero_own), and they poll the flag of the
// CTA that zeroes this CTA's leading row-block (then arrive on zero_ok). The
// epilogue only waits on those shared-memory barriers.
__device__ __forceinline__ void shared_rows_role(const Params& p, int64_t g0, int64_t g1, int lane, uint64_t* zero_own,
                                                 uint64_t* zero_ok) {
  if (p.accumulate) return;
  pdl_wait();  // y: the previous kernel may still use it
  const int b = blockIdx.x;
  const int64_t rl = (g1 - 1) / p.n_cp;  // row-block of the last chunk
  if (rl * p.n_cp >= g0 && (rl + 1) * p.n_cp > g1) {
    const Mat& mt = p.mats[find_mat(p, (int)rl)];
    const int grow0 = ((int)rl - mt.rb0) * 128;
    for (int r = lane - 1; r < 128; r += 31)
      if (grow0 + r < mt.n_rows)
        for (int t = 0; t < p.batch; ++t) mt.y[(int64_t)t * mt.ldy + grow0 + r] = 0.f;
    __threadfence();
    __syncwarp(0xfffffffeu);
    if (lane == 1) {
      st_release_u64(&p.zflags[b], p.epoch);
      mbar_arrive(zero_own);
    }
  }
  const int64_t rf = g0 / p.n_cp;  // row-block of the first chunk
  if (rf * p.n_cp < g0 && lane == 1) {  // it started in an earlier CTA, which zeroes it
    const unsigned long long* fl = &p.zflags[cta_of(p, rf * p.n_cp)];
    const uint64_t t0 = globaltimer_ns();
    while (ld_volatile_u64(fl) != p.epoch) {
      if (*(volatile int*)&g_sg_error != 0 || globaltimer_ns() - t0 > SG_WAIT_NS) {
        sg_set_error(SG_DEVERR_WAIT_TIMEOUT | 0x2D);
        break;
      }
    }
    __threadfence();  // with the flag read: the zeroing happens before the adds
    mbar_arrive(zero_ok);
  }
}

// A segment shared with an earlier CTA (at most the CTA's first one) waits
// for that CTA's zeroing; rather than stall the pipeline at its end, its sums
// are held in registers and reduced after the CTA's last piece.
template <int BT>
struct HeldSegment {
  float v[BT];
  float* y = nullptr;
  int64_t ldy = 0;
  bool on = false;
};

// After the piece of cnt chunks at the cursor: if it ends a segment, write
// acc (lanes with writer set), or hold it, and clear it. Warp-collective.
template <int BT>
__device__ __forceinline__ void end_segment(const Params& p, const Cursor& cur, int cnt, int64_t g0, int row, bool writer,
                                            float (&acc)[BT], HeldSegment<BT>& held, uint64_t* zero_own) {
  const bool rb_end = cur.c + cnt == p.n_ch;
  if (!rb_end && cur.g + cnt != cur.g1) return;
  const Mat& mt = p.mats[cur.mi];
  const int grow = cur.rb * 128 + row;
  const bool live = writer && grow < mt.n_rows;
  const int64_t gr0 = (int64_t)cur.rbg * p.n_cp;
  if (rb_end && gr0 >= g0) {  // this CTA ran the row-block from chunk 0
    if (live) {
#pragma unroll
      for (int t = 0; t < BT; ++t) {
        if (t < p.batch) {
          float* yp = mt.y + (int64_t)t * mt.ldy + grow;
          *yp = p.accumulate ? *yp + acc[t] : acc[t];
        }
      }
    }
  } else if (!p.accumulate && cta_of(p, gr0) != (int)blockIdx.x) {
    held.on = true;
    held.y = live ? mt.y + grow : nullptr;
    held.ldy = mt.ldy;
#pragma unroll
    for (int t = 0; t < BT; ++t) held.v[t] = acc[t];
  } else {
    // accumulate, or this CTA's own trailing row-block: zeroed by warp 0
    const bool ok = p.accumulate || __all_sync(0xffffffffu, mbar_wait(zero_own, 0, 0x2E));
    if (live && ok) {
#pragma unroll
      for (int t = 0; t < BT; ++t)
        if (t < p.batch) red_add_f32(mt.y + (int64_t)t * mt.ldy + grow, acc[t]);
    }
  }
#pragma unroll
  for (int t = 0; t < BT; ++t) acc[t] = 0.f;
}

// the held segment, once the earlier CTA has zeroed its rows. Warp-collective.
template <int BT>
__device__ __forceinline__ void flush_held(const Params& p, const HeldSegment<BT>& held, uint64_t* zero_ok) {
  if (!held.on) return;
  const bool ok = __all_sync(0xffffffffu, mbar_wait(zero_ok, 0, 0x2F));
  if (held.y && ok) {
#pragma unroll
    for (int t = 0; t < BT; ++t)
      if (t < p.batch) red_add_f32(held.y + (int64_t)t * held.ldy, held.v[t]);
  }
}

// ------------------------------------------------------ activation images
// gemv_xprep_kernel: the activation units of one call, in the exact shared-
// memory layout of a unit (block-diagonal tiles with position chunk % GC,
// then sums and scales), written once to global memory for every CTA to
// copy. One warp per (unit, token column t < BT); it writes every row of its
// token in the unit's four tiles (digits in the (position, block) row's
// half, zeros elsewhere), the token-0 warp also the padding rows, so no
// byte of a previous call's image survives. Columns t >= batch are zero.
template <int BT>
__global__ void __launch_bounds__(128) gemv_xprep_kernel(Params p, int n_units) {
  using C = Cfg<BT>;
  pdl_launch_dependents();
  pdl_wait();  // x may come from the previous kernel, which may also still read the images
  const int lane = threadIdx.x & 31;
  const int wg = blockIdx.x * 4 + (threadIdx.x >> 5);
  if (wg >= n_units * BT) return;
  const int u = wg / BT, t = wg - u * BT;
  uint8_t* unit = p.ximg + (int64_t)u * C::XU;
  float v[8];
  load_x8(p, u, t, lane, v);  // zeros for t >= batch and K beyond the matrix
  const UnitDigits ud = unit_digits(v);
  const int c = lane >> 3, j = (lane >> 2) & 1, w = lane & 3;
  uint8_t* tile = unit + c * C::T;
  const int seg = 2 * j + (w >> 1), off = 8 * (w & 1);  // this lane's 8 bytes of a row: half j, word w
#pragma unroll
  for (int k = 0; k < C::GC; ++k)
#pragma unroll
    for (int jj = 0; jj < 2; ++jj)
#pragma unroll
      for (int d = 0; d < 3; ++d) {
        const int n = brow<BT>(k, jj, d, t);
        const bool mine = k == c % C::GC && jj == j;
        *reinterpret_cast<uint2*>(tile + sw64_off(n, seg) + off) =
            mine ? make_uint2(ud.dig[d][0], ud.dig[d][1]) : make_uint2(0u, 0u);
      }
  if (t == 0)
    for (int n = C::ROWS; n < C::N; ++n) *reinterpret_cast<uint2*>(tile + sw64_off(n, seg) + off) = make_uint2(0u, 0u);
  if (t < p.batch) store_tail(reinterpret_cast<float*>(unit + kUC * C::T), ud, t, lane);  // warp-uniform
}

// ---------------------------------------------------------------- GEMV
// BT: live token columns rounded up to a power of two
template <int DT, int BT>
__global__ void __launch_bounds__(Cfg<BT>::THREADS) __maxnreg__(Cfg<BT>::MAXREG) gemv_kernel(Params p) {
  using C = Cfg<BT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  // per group g: a_full[g % SA] -- its A tiles and scale words are in TMEM;
  // a_free[g % SA] and d_full[g % SD] -- its MMAs completed; d_free[g % SD]
  // -- its epilogue is done with the accumulators and scale words
  __shared__ __align__(8) uint64_t w_full[C::RW], w_empty[C::RW], x_full[C::RX], x_empty[C::RX], a_full[C::SA],
      a_free[C::SA], d_full[C::SD], d_free[C::SD], zero_own, zero_ok;
  // two epilogue sets: at a segment end the set that did not run its last
  // piece hands its sums over (seg_full), the other adds them (seg_empty)
  __shared__ __align__(8) uint64_t seg_full, seg_empty;
  __shared__ float seg_acc[C::NSET == 2 ? 128 * BT : 1];
  __shared__ uint32_t tmem_base_sh;

  pdl_launch_dependents();  // the next kernel may start its own prologue once SMs free up
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int64_t g0, g1;
  cta_range(p, blockIdx.x, g0, g1);

  if (threadIdx.x == 0) {
    for (int r = 0; r < C::RW; ++r) {
      mbar_init(&w_full[r], 1);
      mbar_init(&w_empty[r], 4);
    }
    for (int r = 0; r < C::RX; ++r) {
      mbar_init(&x_full[r], C::XPP);
      mbar_init(&x_empty[r], 4);
    }
    for (int s = 0; s < C::SA; ++s) {
      mbar_init(&a_full[s], 4);
      mbar_init(&a_free[s], 1);
    }
    for (int s = 0; s < C::SD; ++s) {
      mbar_init(&d_full[s], 1);
      mbar_init(&d_free[s], 4);
    }
    mbar_init(&zero_own, 1);
    mbar_init(&zero_ok, 1);
    mbar_init(&seg_full, 4);
    mbar_init(&seg_empty, 4);
    mbar_fence_init();
  }
  // activation tiles built here: zero once; afterwards only digit bytes are written
  if (!C::XPRE)
    for (int i = threadIdx.x; i < C::RX * C::XU / 16; i += C::THREADS)
      reinterpret_cast<uint4*>(smem + C::OFF_X)[i] = make_uint4(0u, 0u, 0u, 0u);
  if (warp == 1) sg_tmem_alloc(&tmem_base_sh, C::TMEM_COLS);
  sg_tc_fence_before();
  __syncthreads();
  sg_tc_fence_after();
  const uint32_t tmem = tmem_base_sh;

  if (warp == 0) {
    // ========================================================= weight producer
    if (lane == 0) {
      Cursor cur;
      cur.init(p, g0, g1);
      int v = 0;
      Ring<C::RW> wr;
      for (; cur.more(); ++v, wr.next(), cur.next(p)) {
        const int ws = wr.slot;
        if (v >= C::RW && !mbar_wait(&w_empty[ws], wr.phase ^ 1u, 0x21)) break;
        const Mat& mt = p.mats[cur.mi];
        const int cnt = cur.cnt(p);
        uint8_t* dst = smem + C::OFF_W + ws * kWU;
        mbar_arrive_expect_tx(&w_full[ws], cnt * SG_TILE_BYTES + (DT == SG_DTYPE_Q4_K ? 512 : 0));
        bulk_g2s(dst, mt.tiles + ((int64_t)cur.rb * p.n_ch + cur.c) * SG_TILE_BYTES, cnt * SG_TILE_BYTES, &w_full[ws]);
        if (DT == SG_DTYPE_Q4_K)  // the unit's Q4_K super-block scales
          bulk_g2s(dst + kUC * SG_TILE_BYTES, mt.dd + ((int64_t)cur.rb * mt.n_sb + cur.sc()) * 128, 512, &w_full[ws]);
      }
      if (*(volatile int*)&g_sg_error != 0)  // error path: no copy may land after the CTA exits
        for (int j = max(0, v - C::RW); j < v; ++j) mbar_wait_drain(&w_full[j % C::RW], (j / C::RW) & 1);
    } else {
      shared_rows_role(p, g0, g1, lane, &zero_own, &zero_ok);
    }
  } else if (warp == 1 || (C::NSET == 2 && warp == C::MMA1_WARP)) {
    // ============================================================ MMA issuers
    if (lane == 0) {
      const int set = warp == 1 ? 0 : 1;
      Cursor cur;
      cur.init(p, g0, g1);
      if (set == 1 && cur.more()) cur.next(p);
      int g = 0, last_sd = 0;
      uint32_t last_ph = 0u;
      bool ok = true;
      Ring<C::RX, C::NSET> xr(set);
      Ring<C::SA, C::NSET> ar(set);
      Ring<C::SD, C::NSET> dr(set);
      while (cur.more() && ok) {
        const int xs = xr.slot, cnt = cur.cnt(p), ci0 = cur.ci0();
        if (!mbar_wait(&x_full[xs], xr.phase, 0x23)) break;
        const uint64_t xdesc = sg_sdesc(smem_u32(smem + C::OFF_X + xs * C::XU), SG_SW64);
        for (int gi = 0; gi * C::CPG < cnt; ++gi, ++g, ar.next(), dr.next()) {
          const int sa = ar.slot, sd = dr.slot;
          // the dequant warps waited for the accumulator slot's previous
          // epilogue before they signalled a_full: it makes both slots ready
          if (!mbar_wait(&a_full[sa], ar.phase, 0x24)) {
            ok = false;
            break;
          }
          sg_tc_fence_after();
          // The issuing thread is a pacing resource: keep the work between
          // MMAs to a few adds. A descriptor's start-address field is the
          // byte address / 16, so a tile offset is added to it directly
          // (shared memory addresses stay below 2^18: no carry).
          const int gc = min(C::CPG, cnt - gi * C::CPG);
          const uint32_t dbase = tmem + C::d_col(sd), abase = tmem + C::a_col(sa);
          const uint64_t bdesc = xdesc + (uint64_t)(((ci0 + gi * C::CPG) * C::T) >> 4);
#pragma unroll
          for (int ci = 0; ci < C::CPG; ++ci) {
            const uint32_t d = dbase + (uint32_t)((ci / C::GC) * C::N);
            const uint64_t bd = bdesc + (uint64_t)((ci * C::T) >> 4);
            const uint32_t live = ci < gc;
            // one MMA per 32-block: 8 TMEM columns of A, 32 bytes of each B row
            sg_umma_i8_tmem_a_if(d, abase + (uint32_t)(ci * kACols), bd, C::IDESC, ci % C::GC == 0 ? 0u : 1u, live);
            sg_umma_i8_tmem_a_if(d, abase + (uint32_t)(ci * kACols + 8), bd + 2, C::IDESC, 1u, live);
          }
          sg_umma_commit(&d_full[sd]);
          sg_umma_commit(&a_free[sa]);
          last_sd = sd;
          last_ph = dr.phase;
        }
        xr.next();
#pragma unroll
        for (int i = 0; i < C::NSET; ++i)
          if (cur.more()) cur.next(p);
      }
      // every MMA issued must have completed before TMEM is freed (the last
      // commit covers all of them; on the normal path this returns at once)
      if (g > 0) mbar_wait_drain(&d_full[last_sd], last_ph);
    }
  } else if (warp < 6) {
    // ======================================================== dequant warps
    const int row = (warp & 3) * 32 + lane;  // TMEM lane quadrant = warp % 4
    const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    Cursor cur;
    cur.init(p, g0, g1);
    int g = 0;
    bool ok = true;
    Ring<C::RW> wr;
    Ring<C::SA> ar;
    Ring<C::SD> dr;
    for (; cur.more() && ok; wr.next(), cur.next(p)) {
      const int ws = wr.slot, cnt = cur.cnt(p);
      if (!__all_sync(0xffffffffu, mbar_wait(&w_full[ws], wr.phase, 0x26))) break;
      const uint8_t* wu = smem + C::OFF_W + ws * kWU;
      const uint32_t ddw = DT == SG_DTYPE_Q4_K ? *reinterpret_cast<const uint32_t*>(wu + kUC * SG_TILE_BYTES + row * 4) : 0u;
      // A group's words of this row: every chunk slot of the group is read,
      // live or not (a slot past the piece holds stale bytes of the ring and
      // no MMA reads its columns), so the reads are straight-line code.
      uint4 n0[C::CPG], n1[C::CPG];
      uint32_t scw[4] = {0u, 0u, 0u, 0u};
      auto load_group = [&](int gi) {
#pragma unroll
        for (int ci = 0; ci < C::CPG; ++ci) {
          const uint8_t* tile = wu + (gi * C::CPG + ci) * SG_TILE_BYTES;
          n0[ci] = *reinterpret_cast<const uint4*>(tile + row * 16);         // block 0: K 0..31
          n1[ci] = *reinterpret_cast<const uint4*>(tile + 2048 + row * 16);  // block 1: K 32..63
          scw[ci] = *reinterpret_cast<const uint32_t*>(tile + SG_TILE_SC_OFF + row * 4);
        }
      };
      // With one group per piece the words fit in registers: the weight slot
      // is released before the waits for TMEM, so it holds only copies in
      // flight and the ring keeps the HBM stream full.
      constexpr bool kEarly = C::CPG == kUC;
      if (kEarly) {
        load_group(0);
        __syncwarp();
        if (lane == 0) mbar_arrive(&w_empty[ws]);
      }
      for (int gi = 0; gi * C::CPG < cnt; ++gi, ++g, ar.next(), dr.next()) {
        const int sa = ar.slot, sd = dr.slot;
        // the A slot was last read by the MMAs of group g - SA, the scale
        // words and accumulators by the epilogue of group g - SD
        const bool w = (g < C::SA || mbar_wait(&a_free[sa], ar.phase ^ 1u, 0x27)) &&
                       (g < C::SD || mbar_wait(&d_free[sd], dr.phase ^ 1u, 0x28));
        if (!__all_sync(0xffffffffu, w)) {
          ok = false;
          break;
        }
        sg_tc_fence_after();
        if (!kEarly) load_group(gi);
#pragma unroll
        for (int ci = 0; ci < C::CPG; ++ci) {
          const uint32_t nw[8] = {n0[ci].x, n0[ci].y, n0[ci].z, n0[ci].w, n1[ci].x, n1[ci].y, n1[ci].z, n1[ci].w};
          // column 2w: the low nibbles of word w (K offsets 0,4,1,5 of its 8),
          // column 2w+1: the high nibbles (2,6,3,7)
          uint32_t av[16];
#pragma unroll
          for (int jj = 0; jj < 8; ++jj) {
            av[2 * jj] = nw[jj] & 0x0F0F0F0Fu;
            av[2 * jj + 1] = (nw[jj] >> 4) & 0x0F0F0F0Fu;
          }
          sg_tmem_st16(lane_base + C::a_col(sa) + (uint32_t)(ci * kACols), av);
        }
        const uint32_t scc = lane_base + C::sc_col(sd);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint32_t one[1] = {scw[i]};
          sg_tmem_st_n<1>(scc + (uint32_t)i, one);
        }
        const uint32_t ddv[1] = {ddw};
        sg_tmem_st_n<1>(scc + 4, ddv);
        sg_tmem_st_wait();
        sg_tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&a_full[sa]);
      }
      if (!kEarly) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&w_empty[ws]);  // the piece's weights are all in TMEM now
      }
    }
  } else if (C::x_warp(warp) >= 0) {
    // ===================================================== activation warps
    if constexpr (C::XPRE) {
      // the call's unit images are ready once the prep kernel completes: one
      // bulk copy per piece
      if (warp == 10 && lane == 0) {
        pdl_wait();
        Cursor cur;
        cur.init(p, g0, g1);
        int v = 0;
        Ring<C::RX> xr;
        for (; cur.more(); ++v, xr.next(), cur.next(p)) {
          const int xs = xr.slot;
          if (v >= C::RX && !mbar_wait(&x_empty[xs], xr.phase ^ 1u, 0x2A)) break;
          mbar_arrive_expect_tx(&x_full[xs], C::XU);
          bulk_g2s(smem + C::OFF_X + xs * C::XU, p.ximg + (int64_t)cur.sc() * C::XU, C::XU, &x_full[xs]);
        }
        if (*(volatile int*)&g_sg_error != 0)  // error path: no copy may land after the CTA exits
          for (int j = max(0, v - C::RX); j < v; ++j) mbar_wait_drain(&x_full[j % C::RX], (j / C::RX) & 1);
      }
    } else {
    // Warp xw converts token xw % XPP of the pieces v with v % XL == xw / XPP.
    // A job's x (1 KB) is fetched with cp.async into the warp's staging
    // slots XS - 1 jobs ahead, so the global latency overlaps the jobs in
    // between.
    const int xw = C::x_warp(warp);
    constexpr int XS = C::XS, XL = C::XL;
    const int xl = xw / C::XPP, t = xw % C::XPP;
    const bool live = t < p.batch;  // warp-uniform
    float* stage = reinterpret_cast<float*>(smem + C::OFF_S) + xw * XS * 256;
    pdl_wait();  // x may come from the previous kernel
    Cursor cur;
    cur.init(p, g0, g1);
    const int shift0 = cur.ci0() % C::GC;  // only a CTA's first piece can start inside a unit
    for (int i = 0; i < xl && cur.more(); ++i) cur.next(p);
    Cursor pf = cur;  // next piece to stage for this warp
    // stage the job at pf into slot sl (an empty group when pf is done), then
    // step pf to this warp's next job
    auto stage_next = [&](int sl) {
      if (pf.more()) {
        const int k0 = 256 * pf.sc() + 8 * lane;
        if (live) {
          const float* src = p.x + (int64_t)t * p.ldx + (k0 < p.K ? k0 : 0);
          const uint32_t nb = k0 < p.K ? 16u : 0u;  // 0: zero-fill, nothing read
          float* dst = stage + sl * 256 + 8 * lane;
          cp_async16(dst, src, nb);
          cp_async16(dst + 4, src + 4, nb);
        }
#pragma unroll
        for (int i = 0; i < XL; ++i)
          if (pf.more()) pf.next(p);
      }
      cp_async_commit();
    };
#pragma unroll
    for (int j = 0; j < XS - 1; ++j) stage_next(j);
    int job = 0;
    Ring<C::RX, XL> xr(xl);
    for (int v = xl; cur.more(); v += XL) {
      const int xs = xr.slot;
      // the slot was last read by piece v - RX
      if (v >= C::RX && !__all_sync(0xffffffffu, mbar_wait(&x_empty[xs], xr.phase ^ 1u, 0x2A))) break;
      uint8_t* xu = smem + C::OFF_X + xs * C::XU;
      stage_next((job + XS - 1) % XS);
      cp_async_wait<XS - 1>();  // this job's copies have landed (each lane reads only its own)
      const float* sj = stage + (job % XS) * 256 + 8 * lane;
      if (v == C::RX && shift0 != 0 && live) {
        // piece 0 placed its rows at shifted positions: clear every row of
        // this warp's token in the slot
        for (int e = lane; e < kUC * C::GC * 6 * 4; e += 32) {  // (tile, row of the token, 16-byte segment)
          const int c = e / (C::GC * 6 * 4), r = (e / 4) % (C::GC * 6), sgm = e % 4;
          const int n = brow<BT>(r / 6, (r / 3) % 2, r % 3, t);
          reinterpret_cast<uint4*>(xu + c * C::T + n * 64)[sgm] = make_uint4(0u, 0u, 0u, 0u);
        }
        __syncwarp();
      }
      if (live) {
        const float4 a = *reinterpret_cast<const float4*>(sj);
        const float4 b = *reinterpret_cast<const float4*>(sj + 4);
        const float xv[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
        store_digits<BT>(xu, unit_digits(xv), t, lane, cur.ci0());
      }
      ++job;
      fence_proxy_async_smem();  // the tensor core reads the tiles through the async proxy
      __syncwarp();
      if (lane == 0) mbar_arrive(&x_full[xs]);
      xr.next();
#pragma unroll
      for (int i = 0; i < XL; ++i)
        if (cur.more()) cur.next(p);
    }
    cp_async_wait<0>();  // no copy may land after the CTA exits
    }
  } else if ((warp >= 6 && warp < 10) || (C::NSET == 2 && warp >= 12 && warp < 16)) {
    // ============================================================ epilogue warps
    // warps 6-9 (set 0) and, with two sets, 12-15 (set 1); set s runs the
    // pieces v with v % NSET == s and sums them per row; at a segment end the
    // other set's sums are added in before the store
    const int set = warp >= 12 ? 1 : 0;
    const int q = warp & 3;  // TMEM lane quadrant
    const int row = q * 32 + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
    pdl_wait();  // y: the previous kernel may still use it
    HeldSegment<BT> held;
    float acc[BT];
#pragma unroll
    for (int t = 0; t < BT; ++t) acc[t] = 0.f;
    Cursor cur;
    cur.init(p, g0, g1);
    bool ok = true;
    Ring<C::RX, C::NSET> xr(set);
    Ring<C::SD, C::NSET> dr(set);
    int segs = 0;  // segment ends passed (both sets count every one)
    for (int v = 0; cur.more() && ok; ++v, cur.next(p)) {
      const int cnt = cur.cnt(p), ci0 = cur.ci0();
      if (C::NSET == 2 && (v & 1) != set) {
        if (cur.c + cnt == p.n_ch || cur.g + cnt == cur.g1) {
          // the other set ends this segment: hand it this set's sums
          if (segs > 0 && !__all_sync(0xffffffffu, mbar_wait(&seg_empty, (segs - 1) & 1, 0x30))) break;
#pragma unroll
          for (int t = 0; t < BT; ++t) {
            seg_acc[row * BT + t] = acc[t];
            acc[t] = 0.f;
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&seg_full);
          ++segs;
        }
        continue;
      }
      const int xs = xr.slot;
      if (!__all_sync(0xffffffffu, mbar_wait(&x_full[xs], xr.phase, 0x2B))) break;
      const float* tail = reinterpret_cast<const float*>(smem + C::OFF_X + xs * C::XU + kUC * C::T);
      float accu[BT];
#pragma unroll
      for (int t = 0; t < BT; ++t) accu[t] = 0.f;
      for (int gi = 0; gi * C::CPG < cnt; ++gi, dr.next()) {
        const int sd = dr.slot;
        if (!__all_sync(0xffffffffu, mbar_wait(&d_full[sd], dr.phase, 0x25))) {
          ok = false;
          break;
        }
        sg_tc_fence_after();
        const int gc = min(C::CPG, cnt - gi * C::CPG);
        uint32_t scw[4], ddv[1];
        const uint32_t scc = lane_base + C::sc_col(sd);
#pragma unroll
        for (int i = 0; i < 4; ++i) sg_tmem_ld_n<1>(scc + (uint32_t)i, *reinterpret_cast<uint32_t(*)[1]>(&scw[i]));
        sg_tmem_ld_n<1>(scc + 4, ddv);
        float dmx = 0.f, dmy = 0.f;
#pragma unroll
        for (int a = 0; a < C::NACC; ++a) {
          if (a * C::GC >= gc) break;  // warp-uniform
          const uint32_t abase = lane_base + C::d_col(sd) + (uint32_t)(a * C::N);
          uint32_t dv[C::LC];
#pragma unroll
          for (int kb = 0; kb < 2 * C::GC; ++kb) {
            // (position k, block blk): columns brow(k, blk, d, t) = kb*3*BT + d*BT + t
            const int k = kb >> 1, blk = kb & 1, col = kb * 3 * BT;
            if (col % C::LC == 0) {
              tmem_ld_cols<C::LC>(abase + (uint32_t)col, dv);
              sg_tmem_ld_wait();
            }
            if (DT == SG_DTYPE_Q4_K && a == 0 && kb == 0) {
              const float2 dm = __half22float2(*reinterpret_cast<const __half2*>(&ddv[0]));
              dmx = dm.x;
              dmy = dm.y;
            }
            // every position is computed and the dead ones (past the piece:
            // stale accumulator columns) are dropped by a select
            const int ci = a * C::GC + k;
            const bool live = ci < gc;
            const int cu = (ci0 + gi * C::CPG + ci) & 3;  // chunk within the unit
            const uint32_t w = scw[ci];
            float sc, of;
            if (DT == SG_DTYPE_Q4_0) {
              sc = __half2float(__ushort_as_half((unsigned short)(w >> (16 * blk))));
              of = 0.f;
            } else {
              sc = dmx * (float)((w >> (8 * blk)) & 0xFFu);
              of = dmy * (float)((w >> (16 + 8 * blk)) & 0xFFu);
            }
            const float* sv = tail + kSumOff / 4 + (cu * 2 + blk) * 16;
            const int c0 = col % C::LC;
#pragma unroll
            for (int t = 0; t < BT; ++t) {
              const float dot = digit_dot(dv[c0 + t], dv[c0 + BT + t], dv[c0 + 2 * BT + t]);
              const float nv = DT == SG_DTYPE_Q4_0 ? fmaf(sc, fmaf(-8.f, sv[t], dot), accu[t])
                                                   : fmaf(sc, dot, fmaf(-of, sv[t], accu[t]));
              accu[t] = live ? nv : accu[t];
            }
          }
        }
        sg_tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&d_free[sd]);
      }
      if (!ok) break;
#pragma unroll
      for (int t = 0; t < BT; ++t) acc[t] = fmaf(accu[t], tail[kInvOff / 4 + t], acc[t]);
      __syncwarp();
      if (lane == 0) mbar_arrive(&x_empty[xs]);  // this warp is done with the unit's sums and scales
      xr.next();
      if (C::NSET == 2 && (cur.c + cnt == p.n_ch || cur.g + cnt == cur.g1)) {
        if (!__all_sync(0xffffffffu, mbar_wait(&seg_full, segs & 1, 0x31))) break;
#pragma unroll
        for (int t = 0; t < BT; ++t) acc[t] += seg_acc[row * BT + t];
        __syncwarp();
        if (lane == 0) mbar_arrive(&seg_empty);
        ++segs;
      }
      end_segment<BT>(p, cur, cnt, g0, row, true, acc, held, &zero_own);
    }
    flush_held<BT>(p, held, &zero_ok);
  }
  sg_tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    sg_tc_fence_after();
    sg_tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// ------------------------------------------------------------ host side
constexpr size_t kFlagsBytes = (size_t)kMaxCtas * sizeof(unsigned long long);  // workspace: zeroing flags, then images

template <int DT, int BT>
cudaError_t launch(Params p, int rb_total, int num_sms, cudaStream_t st) {
  using C = Cfg<BT>;
  p.spl = C::SPL;
  p.n_cp = (p.n_ch + C::SPL - 1) / C::SPL * C::SPL;
  p.total = (int64_t)rb_total * p.n_cp;
  if (p.total >= INT_MAX / 2) return cudaErrorInvalidValue;  // the device cursor counts chunks in 32 bits
  const int64_t slots = p.total / p.spl;
  const int G = (int)std::max<int64_t>(1, std::min<int64_t>(std::min(num_sms * C::CPS, kMaxCtas), slots));
  static int attr_done[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_done[dev]) {
    const cudaError_t e = cudaFuncSetAttribute(gemv_kernel<DT, BT>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return e;
    attr_done[dev] = 1;
  }
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = sg_pdl_enabled() ? 1 : 0;
  if (C::XPRE) {
    const int n_units = (p.n_ch + kUC - 1) / kUC;
    cudaLaunchConfig_t x = {};
    x.gridDim = dim3((unsigned)((n_units * BT + 3) / 4));
    x.blockDim = dim3(128);
    x.stream = st;
    x.attrs = attr;
    x.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&x, gemv_xprep_kernel<BT>, p, n_units);
    if (e != cudaSuccess) return e;
  }
  cudaLaunchConfig_t g = {};
  g.gridDim = dim3((unsigned)G);
  g.blockDim = dim3(C::THREADS);
  g.dynamicSmemBytes = C::SMEM;
  g.stream = st;
  g.attrs = attr;
  g.numAttrs = 1;
  return cudaLaunchKernelEx(&g, gemv_kernel<DT, BT>, p);
}

}  // namespace gemv_tc

size_t sg_gemv_scratch_bytes(int64_t n_cols, int batch) {
  using namespace gemv_tc;
  const int64_t n_units = ((n_cols + 63) / 64 + kUC - 1) / kUC;
  const size_t xu = batch <= 2 ? 0 : batch <= 4 ? Cfg<4>::XU : batch <= 8 ? Cfg<8>::XU : Cfg<16>::XU;
  return kFlagsBytes + (size_t)n_units * xu;
}

cudaError_t sg_gemv(const SgGemvMat* mats, int n_mats, const float* x, int64_t ldx, int batch, bool accumulate,
                    void* scratch, size_t scratch_bytes, int num_sms, cudaStream_t st) {
  using namespace gemv_tc;
  if (n_mats < 1 || n_mats > SG_GEMV_MAX_MATS || batch < 1 || batch > SG_GEMV_MAX_BATCH || !x || !scratch)
    return cudaErrorInvalidValue;
  const SgDevWeight* w0 = mats[0].w;
  const int64_t K = w0->n_cols;
  if ((K & 31) || K > (1 << 28) || ((uintptr_t)x & 15) || (ldx & 3) || ldx < K) return cudaErrorInvalidValue;
  if (scratch_bytes < sg_gemv_scratch_bytes(K, batch) || ((uintptr_t)scratch & 255)) return cudaErrorInvalidValue;
  Params p = {};
  p.n_mats = n_mats;
  p.batch = batch;
  p.n_ch = (int)w0->n_ch;
  p.accumulate = accumulate ? 1 : 0;
  int rb = 0;
  for (int i = 0; i < n_mats; ++i) {
    const SgDevWeight* w = mats[i].w;
    if (w->n_cols != K || w->dtype != w0->dtype || !mats[i].y || mats[i].ldy < w->n_rows) return cudaErrorInvalidValue;
    p.mats[i] = {w->tiles, w->dd, mats[i].y, mats[i].ldy, (int)w->n_rb, (int)w->n_rows, (int)w->n_sb, rb};
    rb += (int)w->n_rb;
  }
  p.x = x;
  p.ldx = ldx;
  p.K = (int)K;
  p.zflags = static_cast<unsigned long long*>(scratch);
  p.ximg = static_cast<uint8_t*>(scratch) + kFlagsBytes;
  static std::atomic<unsigned long long> epochs{1};
  p.epoch = epochs.fetch_add(1);
#define SG_GEMV_LAUNCH(DT)                                                           \
  switch (batch <= 1 ? 1 : batch <= 2 ? 2 : batch <= 4 ? 4 : batch <= 8 ? 8 : 16) { \
    case 1: return launch<DT, 1>(p, rb, num_sms, st);                                \
    case 2: return launch<DT, 2>(p, rb, num_sms, st);                                \
    case 4: return launch<DT, 4>(p, rb, num_sms, st);                                \
    case 8: return launch<DT, 8>(p, rb, num_sms, st);                                \
    default: return launch<DT, 16>(p, rb, num_sms, st);                              \
  }
  if (w0->dtype == SG_DTYPE_Q4_0) SG_GEMV_LAUNCH(SG_DTYPE_Q4_0)
  SG_GEMV_LAUNCH(SG_DTYPE_Q4_K)
#undef SG_GEMV_LAUNCH
}
