/*
 * Plain-C restatement of DeepSeek-V3 no-aux routing, TEST INFRASTRUCTURE ONLY
 * (the checker for the GPU routing kernel; never linked into the product).
 *
 * Follows the routing step of the operator definition's reference
 * (resources/moe_fp8_block_scale_ds_routing_topk8_ng8_kg4_e32_h7168_i2048.json:146,
 * "2) No-aux routing"), one token at a time with scalar fp32 arithmetic:
 *   s = 1 / (1 + exp(-x)), sb = s + bias
 *   group score = sum of the two largest sb in each group of 32 experts
 *   keep the 4 groups with the largest scores (ties: lower group index)
 *   select the 8 largest sb among kept experts (ties: lower expert index)
 *   w = s / (sum of the 8 selected s + 1e-20) * scale
 * Outputs are in selection order (descending sb).
 */
#include <math.h>
#include <stdint.h>

#define N_EXPERTS 256
#define N_GROUPS 8
#define GROUP_SIZE 32
#define TOPK_GROUPS 4
#define TOPK 8

static float sigmoidf_ref(float x) { return 1.0f / (1.0f + expf(-x)); }

void route_tokens(const float* logits, const float* bias, int T, float scale, int32_t* topk_idx, float* topk_w) {
  for (int t = 0; t < T; ++t) {
    const float* x = logits + (long)t * N_EXPERTS;
    float s[N_EXPERTS], sb[N_EXPERTS];
    for (int e = 0; e < N_EXPERTS; ++e) {
      s[e] = sigmoidf_ref(x[e]);
      sb[e] = s[e] + (bias ? bias[e] : 0.0f);
    }
    float gs[N_GROUPS];
    for (int g = 0; g < N_GROUPS; ++g) {
      float m1 = -INFINITY, m2 = -INFINITY;
      for (int j = 0; j < GROUP_SIZE; ++j) {
        float v = sb[g * GROUP_SIZE + j];
        if (v > m1) { m2 = m1; m1 = v; }
        else if (v > m2) { m2 = v; }
      }
      gs[g] = m1 + m2;
    }
    int keep[N_GROUPS];
    for (int g = 0; g < N_GROUPS; ++g) {
      int rank = 0;
      for (int h = 0; h < N_GROUPS; ++h) rank += (gs[h] > gs[g]) || (gs[h] == gs[g] && h < g);
      keep[g] = rank < TOPK_GROUPS;
    }
    int taken[N_EXPERTS] = {0};
    float ssel[TOPK];
    for (int k = 0; k < TOPK; ++k) {
      int best = -1;
      for (int e = 0; e < N_EXPERTS; ++e) {
        if (!keep[e / GROUP_SIZE] || taken[e]) continue;
        if (best < 0 || sb[e] > sb[best]) best = e;
      }
      taken[best] = 1;
      topk_idx[(long)t * TOPK + k] = best;
      ssel[k] = s[best];
    }
    float sum = 0.0f;
    for (int k = 0; k < TOPK; ++k) sum += ssel[k];
    for (int k = 0; k < TOPK; ++k) topk_w[(long)t * TOPK + k] = (ssel[k] / (sum + 1e-20f)) * scale;
  }
}
