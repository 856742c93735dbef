// Standalone glue kernels, dequantisation and argmax.  See glue.cu.
#pragma once
#include "common.cuh"

namespace sb {

int norm_rows_launch(const uint16_t* x, const int64_t* ids, const uint16_t* embed, int embed_rows, float mult,
                     const uint16_t* w, uint16_t* y, uint16_t* h_out, int rows, int n, float eps, bool pdl,
                     cudaStream_t s);
int dequant_launch(const SbLinear& lin, void* out, bool f32, cudaStream_t s);
int rmsnorm_launch(const uint16_t* x, const uint16_t* w, uint16_t* y, int rows, int n, float eps, cudaStream_t s);
int silu_mul_launch(const uint16_t* g, const uint16_t* u, uint16_t* o, int64_t count, cudaStream_t s);
int set_ctrl_launch(int32_t* ctrl, int slot, int padlen, cudaStream_t s);
int residual_launch(const uint16_t* x, const uint16_t* y, uint16_t* z, int64_t count, float alpha, cudaStream_t s);
int rope_launch(uint16_t* x, int rows, int heads, const int32_t* pos, const uint16_t* cs, const uint16_t* sn,
                cudaStream_t s);
int argmax_launch(const uint16_t* x, int rows, int n, int64_t* out, cudaStream_t s);

}  // namespace sb
