// gsv_sampler.h -- sampler settings of the AR path.
//
// Same struct, fields and defaults as gsv.cpp's src/gsv_sampler.h:18-23 (the TTS.py inference
// defaults), so gsv_ar.h is source-compatible with the reference callers. Inside the reference tree
// the reference's own header (which also declares its host sampler) is used instead of this one.
#pragma once

#include <cstdint>

struct gsv_sampler_cfg {
    int top_k = 15;                    // <= 0 disables top-k
    float top_p = 1.0f;                // >= 1 disables nucleus filtering
    float temperature = 1.0f;
    float repetition_penalty = 1.35f;
};
