/* Minimal stand-in for ggml.h so the reference's MoE sources compile without the
 * (absent, unpinned) ggml submodule.  The reference uses ggml only for the
 * ggml_type enum (src/hunyuan_model.h:3,54) and two opaque forward declarations
 * (src/hunyuan_model.h:71-75).  Enum values follow the GGUF specification.
 * Test infrastructure only: never linked into the product library. */
#pragma once
enum ggml_type { GGML_TYPE_F32 = 0, GGML_TYPE_F16 = 1, GGML_TYPE_Q4_0 = 2, GGML_TYPE_Q8_0 = 8 };
struct ggml_context;
struct ggml_tensor;
