/*
 * minima_forward.h — the drop-in replacement of the Minima reference's
 * forward.h (forward.h:43-57), implemented by minima_b200/host/forward_cuda.c
 * (libminima_forward.so) over the device path of minima_cuda.h.
 *
 * Same functions, signatures and return conventions as forward.c:
 *   activations_init  <- forward.h:43-44 (forward.c:124-170): the same
 *                        buffers, carved from the caller's arena in the same
 *                        order, so code that reads Activations (the
 *                        reference's backward.c, its tests) sees the layout it
 *                        expects.
 *   rmsnorm, silu     <- forward.h:47-48, 51 (forward.c:13-22, 58-60): scalar
 *                        helpers of the training code, host arithmetic in the
 *                        reference's order.
 *   matmul            <- forward.h:49-50 (forward.c:24-40): on the device
 *                        (mc_matmul), fp32, k ascending per output.
 *   model_forward     <- forward.h:56-57 (forward.c:176-274): the batched
 *                        causal forward on the device (mc_model_forward_caches)
 *                        writing the logits and every cache model_backward
 *                        reads into the caller's Activations; NULL on invalid
 *                        dimensions or token ids, as forward.c:179-186.
 * Inside a Minima tree, MINIMA_REFERENCE_HEADERS makes the reference's own
 * headers provide the types.
 */
#ifndef MINIMA_FORWARD_H
#define MINIMA_FORWARD_H

#include "minima_generate.h"

#ifndef MINIMA_REFERENCE_HEADERS
#ifdef __cplusplus
extern "C" {
#endif

/* forward.h:43-44 */
bool activations_init(Activations* act, Arena* temp_arena, int batch, int seq, const Model* model);
/* forward.h:47-48 */
void rmsnorm(float* out, const float* x, const float* scale, int dim, float eps);
/* forward.h:49-50 */
void matmul(float* out, const float* x, const float* w, int n, int d_in, int d_out);
/* forward.h:51 */
float silu(float x);
/* forward.h:56-57 */
float* model_forward(Model* model, Activations* act, const uint16_t* tokens, int batch, int seq);

#ifdef __cplusplus
}
#endif
#endif /* MINIMA_REFERENCE_HEADERS */
#endif
