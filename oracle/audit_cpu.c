/*
 * audit_cpu.c -- TEST INFRASTRUCTURE ONLY: a C restatement of the reference audit kernel, used as the
 * timed CPU baseline of bench.py and checked against the numpy oracle (oracle/audit.py) by the tests.
 *
 * It restates tile_lse_kernel (runtime/audit_kernel.py:34-109) as launched by RecordingPlane.launch
 * (:224-265): for every selected row and every tile of tile_blocks*block_size tokens whose first token
 * lies below the row's length, m = max_j q.k_j*scale and l = sum_j exp(q.k_j*scale - m) over the
 * tile's tokens below the length, for the G query rows of KV head `group`, stored into every block
 * cell of the tile that starts below the length. Float32 arithmetic on exactly upcast fp16/bf16 input.
 * Tiles are independent, so they are spread over OpenMP threads.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

static inline float bf16_to_f32(uint16_t x) {
  uint32_t u = (uint32_t)x << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static inline float f16_to_f32(uint16_t x) {
  _Float16 h;
  memcpy(&h, &x, 2);
  return (float)h;
}

int ekv_oracle_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* dtype: 0 = fp16, 1 = bf16. Strides in elements. lse: [2][layers][rows][width][G]. */
void ekv_oracle_tile_lse(const uint16_t* q, const uint16_t* k, int dtype, const int32_t* table,
                         const int32_t* lens, const int32_t* qrow, const uint8_t* select, int flag,
                         float* lse, float scale, int layer, int group, int64_t q_s0, int64_t q_s1,
                         int64_t k_s0, int64_t k_s1, int64_t k_s2, int64_t table_s0, int layers,
                         int rows, int width, int G, int block_size, int tile_blocks, int head_dim,
                         int threads) {
  if (!flag) return;
  const int tt = tile_blocks * block_size;
  const int tiles = (width + tile_blocks - 1) / tile_blocks;
  const int64_t plane = (int64_t)layers * rows * width * G;
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#pragma omp parallel for schedule(dynamic, 4)
#endif
  for (int64_t item = 0; item < (int64_t)rows * tiles; ++item) {
    const int row = (int)(item / tiles), tile = (int)(item % tiles);
    if (!select[row]) continue;
    const int length = lens[row];
    const int first = tile * tt;
    if (first >= length) continue;
    float qf[16][256];
    float score[16][128];
    for (int g = 0; g < G; ++g) {
      const uint16_t* src = q + (int64_t)qrow[row] * q_s0 + (int64_t)(group * G + g) * q_s1;
      for (int d = 0; d < head_dim; ++d) qf[g][d] = dtype ? bf16_to_f32(src[d]) : f16_to_f32(src[d]);
    }
    for (int t = 0; t < tt; ++t) {
      const int pos = first + t;
      if (pos >= length) {
        for (int g = 0; g < G; ++g) score[g][t] = -INFINITY;
        continue;
      }
      const int32_t block = table[(int64_t)row * table_s0 + pos / block_size];
      const uint16_t* kr = k + (int64_t)block * k_s0 + (int64_t)(pos % block_size) * k_s1 + (int64_t)group * k_s2;
      float kf[256];
      for (int d = 0; d < head_dim; ++d) kf[d] = dtype ? bf16_to_f32(kr[d]) : f16_to_f32(kr[d]);
      for (int g = 0; g < G; ++g) {
        float acc = 0.f;
        for (int d = 0; d < head_dim; ++d) acc += qf[g][d] * kf[d];
        score[g][t] = acc * scale;
      }
    }
    for (int g = 0; g < G; ++g) {
      float peak = -INFINITY;
      for (int t = 0; t < tt; ++t) peak = score[g][t] > peak ? score[g][t] : peak;
      float total = 0.f;
      for (int t = 0; t < tt; ++t) total += expf(score[g][t] - peak);
      for (int i = 0; i < tile_blocks; ++i) {
        const int b = tile * tile_blocks + i;
        if ((int64_t)b * block_size >= length) continue;
        float* cell = lse + (((int64_t)layer * rows + row) * width + b) * G + g;
        cell[0] = peak;
        cell[plane] = total;
      }
    }
  }
}
