// Interface of the fused verify forward (fused_step.cuh, compiled into
// model.cu): the phases of one persistent cooperative launch over the decoder
// layers of one request.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "model.cuh"

namespace ifr {

// one projection: Y (+)= W f(X) over ncols <= 8 columns (exact activations)
struct FGemv {
    const uint8_t *W;       // M-tiles (tiles.cuh)
    int64_t M, K;
    int nrb, nu, fmt, nt;   // row blocks, units, GGML type, column tiles (1: <= 4 columns, 2: <= 8)
    int xf;                 // 0 none, 3 RMSNorm(x, xw, eps) folded into the epilogue
    int ep;                 // 0 store, 1 silu(gate) * up, 2 gelu_tanh(gate) * up (interleaved 16-row blocks)
    int accumulate;         // 1: Y += W f(X)
    int gran;               // row blocks per scheduling unit (2 with ep: whole gate/up pairs)
    const float *X;
    int64_t ldx;
    int ncols;
    float *Y;
    int64_t ldy;
    const float *xw;
    float eps;
};

// the weights of a later GEMV phase, sent toward L2 at the start of this one
struct FPrefetch {
    const uint8_t *W = nullptr;  // null: none
    int nrb = 0, nu = 0, fmt = 0, gran = 1;
};

struct FPhase {
    // kTestAbsent: CTA 0 leaves the launch without arriving at the barrier
    // after this phase (the failure test: the other CTAs' bounded waits run out)
    enum : int { kNone = 0, kGemv = 1, kSsm = 2, kAttnPart = 3, kAttnCombine = 4, kSsmFinal = 5, kTestAbsent = 9 };
    int kind;
    int nobar;              // 1: the next phase does not read this one's output (no grid barrier)
    int vblocks;            // SSM: heads x row splits; attention: slices x row groups (part) or rows (combine)
    int s_hd, hg, part_smem;
    int tiles_smem;         // GEMV: this CTA's M-tiles arrive by one bulk copy into shared memory
    FPrefetch pf[2];
    FPrefetch tl;           // the next GEMV phase's tiles (tiles_smem), copied once this phase frees the buffer
    float *ssq_part;        // SSM: per (head, split, token) sums of y^2 of the split's rows
    float *rec_stage;       // SSM: this call's replay record, committed by the final phase
    FGemv g;
    SsmArgs s;
    AttnArgs a;
};

constexpr int kFusedSsmSplit = 8;  // row splits of a GatedDeltaNet head in the fused launch

// dynamic shared memory of the fused launch: the M-tile buffer, then the
// phases' work area (fragments, partials, SSM and attention state)
constexpr int kFusedSmem = 220 * 1024;
constexpr int kFusedTileBytes = 64 * 1024;
constexpr int kFusedWorkBytes = kFusedSmem - kFusedTileBytes;

// the CTAs of a fused launch (one per SM)
int fused_ctas();
// phase builders: false when the phase is outside what the fused launch
// covers (format, head dim, shared memory); vblocks / hg / part_smem filled
bool fused_gemv_phase(const FGemv &g, FPhase &ph);
// the GatedDeltaNet step as two phases: the row-split state update and the
// final phase (per-head RMSNorm + gate, conv history / replay commits);
// ssq_part: H * kFusedSsmSplit * 8 floats, rec_stage: H * 8 * (2 hd + 2)
bool fused_ssm_phases(const SsmArgs &a, int head_dim, float *ssq_part, float *rec_stage, FPhase &upd,
                      FPhase &fin);
bool fused_attn_phases(const AttnArgs &a, FPhase &part, FPhase &comb);
// run n phases (device array) as one cooperative launch; ctr: a device
// counter (reset here); a barrier that times out sets the device error flag
// that read_device_error reports; trace (nullable, 4 n (fused_ctas() + 1) + 1
// entries, zeroed by the caller): per phase and CTA the global timer (ns) at
// its start, fragments built, tiles done and phase done; then per phase the
// barrier detail (CTA 0's arrival, target seen, acquire done; the last
// arrival); then CTA 0's end
cudaError_t fused_layers(const FPhase *phases, int n, unsigned *ctr, unsigned long long *trace, cudaStream_t s);
cudaError_t read_fused_error(int *flag, cudaStream_t s);
// the failure test: a two-phase launch in which CTA 0 never arrives at the
// barrier; the other CTAs wait ~2 s, set the error flag and return
cudaError_t fused_absent_cta_test(cudaStream_t s);

}  // namespace ifr
