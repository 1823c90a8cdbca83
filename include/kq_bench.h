/*
 * kq_bench.h -- measurement helpers of libkq.so (not part of the reference-facing interface of
 * kq.h): the roofline denominators that no library reports.
 */
#ifndef KQ_BENCH_H
#define KQ_BENCH_H

#ifdef __cplusplus
extern "C" {
#endif

/* Dense int8 tensor-core throughput of `device`: every SM issues `iters` x 8 back-to-back
 * tcgen05.mma kind::i8 of 128 x 256 x 32 (s32 accumulators in TMEM) from one thread; the best of
 * three timed launches (after one warm-up).  *tops = 2 M N K x MMAs / seconds / 1e12.  Returns 0,
 * or a negative kq_status (-7: the completion wait timed out). */
int kq_measure_int8_tops(int device, int iters, double *tops);

#ifdef __cplusplus
}
#endif
#endif /* KQ_BENCH_H */
