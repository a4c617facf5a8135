// C entry points onto the reference's OWN Euler scheduler — TEST INFRASTRUCTURE ONLY.
//
// Compiled by oracle/build_oracle.py (when the reference tree is present) from the reference's
// header src/infer/scheduler.hpp where it lies, into oracle/_ref/libref_scheduler.so.  The tests
// pin the library's schedule (dlm_sdxl_schedule) and the denoising oracle's arithmetic to the
// reference's EulerDiscreteScheduler: set_timesteps (scheduler.hpp:69-106), scale_model_input
// (:110-119) and the epsilon Euler step (:126-140).
#include <cstring>
#include <exception>

#include "infer/scheduler.hpp"

extern "C" {

// sigmas [steps + 1], timesteps [steps]; returns 0, or -1 when the scheduler rejects `steps`
int ref_sched_set_timesteps(int steps, float* sigmas, float* timesteps) {
  try {
    dollama::EulerDiscreteScheduler s;
    s.set_timesteps(steps);
    std::memcpy(sigmas, s.sigmas().data(), sizeof(float) * (steps + 1));
    std::memcpy(timesteps, s.timesteps().data(), sizeof(float) * steps);
    return 0;
  } catch (const std::exception&) {
    return -1;
  }
}

// scale_model_input at step_index, in place on sample[n]
int ref_sched_scale(int steps, int step_index, float* sample, size_t n) {
  try {
    dollama::EulerDiscreteScheduler s;
    s.set_timesteps(steps);
    s.scale_model_input(sample, n, step_index);
    return 0;
  } catch (const std::exception&) {
    return -1;
  }
}

// one Euler step: prev[n] from model_output[n] and sample[n]
int ref_sched_step(int steps, int step_index, const float* model_output, const float* sample,
                   float* prev, size_t n) {
  try {
    dollama::EulerDiscreteScheduler s;
    s.set_timesteps(steps);
    s.step(model_output, step_index, sample, prev, n);
    return 0;
  } catch (const std::exception&) {
    return -1;
  }
}

}  // extern "C"
