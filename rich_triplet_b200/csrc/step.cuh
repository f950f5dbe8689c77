// step.cuh -- the persistent Gemma 3 decode-step kernel: one cooperative
// launch runs a whole decode step (every layer and the LM head) with one CTA
// per SM and grid-wide barriers between dependent phases.
#pragma once

#include <stdint.h>

#include <cuda_runtime.h>

#include "attention.cuh"
#include "gemv_core.cuh"

namespace rt {

// Shared-memory geometry of the step kernel.
struct StepGeom {
    int warps = 0;     // 0: the shapes do not fit
    int nb = 0;
    int hidden = 0;    // K of the norm prologues
    int kp_max = 0;    // widest Q4_K job input (columns, multiple of 256)
    int kp_lm = 0;     // LM head input (columns, multiple of 128)
    int head_dim = 0;
    int group = 0;     // query heads per KV head
    int njobs = 0;     // projections of a step (4 per layer + the LM head)
    size_t smem = 0;
};

struct StepParams {
    StepGeom geom;
    const gcore::Job* jobs;  // [4 * nlayers + 1]: per layer QKV, O, gate/up, down; then the LM head
    const AttnArgs* attn;    // [nlayers]
    int32_t nlayers;
    uint32_t* sync;          // [0] launches completed (the tags' high bits), [1] CTA exits (zero between launches)
    int* abort;              // set when a CTA gives up; zero between launches
    gcore::SplitScratch scratch;
    int* err;                // error word (kErr*)
    uint64_t* trace;         // [kStepTraceLen] phase timeline of CTA 0 (globaltimer ns), may be null
};

// Timeline slots: layer l, event e (0 QKV prologue done, 1 QKV done, 2
// attention done, 3 O prologue done, 4 O done, 5 gate/up prologue done, 6
// gate/up done, 7 down prologue done, 8 down done) at 1 + 10 l + e; slot 0 =
// kernel start; the last two slots: LM head projection done, token done.
constexpr int kStepTraceLen = 1024;

StepGeom step_geometry(int hidden, int kp_max, int head_dim, int group, int njobs);
// Raise the kernel's shared-memory limit on the current device (outside capture).
cudaError_t step_prepare(const StepGeom& g);
// Cooperative launch of one decode step on `grid` CTAs (one per SM).
cudaError_t step_launch(const StepParams& p, const StepGeom& g, int grid, cudaStream_t s);
// Largest grid that can be co-resident (the kernel needs every CTA at once).
int step_max_grid(const StepGeom& g);

}  // namespace rt
