/*
 * ORACLE - test infrastructure only.  A plain-C restatement of the
 * reference's CPU engine (src/eigen_engine.cpp) used as the parity checker
 * and as the timed CPU baseline.  Nothing in the product links or calls it.
 *
 * Two input/flatten semantics:
 *   ORC_CANONICAL  state element (c, p) at c*HW + p and policy features
 *                  flattened c*HW + p: the network scripts/model.py:48-62
 *                  trains (and the OpenCL / Metal engines compute);
 *   ORC_LITERAL    what src/eigen_engine.cpp does with Eigen's default
 *                  column-major MatrixXf: Map at :211 reads (c, p) from
 *                  c + p*Cin, and the policy Map at :242 flattens c + 2p.
 */
#ifndef EIGEN_RESTATED_H
#define EIGEN_RESTATED_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ORC_CANONICAL 0
#define ORC_LITERAL 1

typedef struct orc_net orc_net;

orc_net* orc_new(void);
void orc_free(orc_net* net);

/* Stores a copy of a named fp32 tensor (the last one of a name wins, as the
 * name map of src/eigen_engine.cpp:23-25). */
int orc_set(orc_net* net, const char* name, const int64_t* dims, int ndims, const float* data);

/* Infers the architecture (src/eigen_engine.cpp:84-95) and folds BN
 * (src/eigen_engine.cpp:52-67).  Returns 0, or -1 with a message in err. */
int orc_finalize(orc_net* net, char* err, int errlen);

int orc_info(const orc_net* net, int* board, int* input_channels, int* filters, int* blocks,
             int* actions);

/* EigenEngine::predict (src/eigen_engine.cpp:205-273) for n positions,
 * split over `threads` POSIX threads (1 = the reference's serial loop,
 * include/inference_engine.h:25-32).  logits may be NULL. */
int orc_predict_batch(const orc_net* net, const float* states, int n, int mode, int threads,
                      float* probs, float* logits, float* values);

#ifdef __cplusplus
}
#endif

#endif
