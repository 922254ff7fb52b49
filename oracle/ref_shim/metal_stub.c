/* Linux has no Metal: the reference never builds ds_metal.m there. These
 * stubs satisfy the symbols ds_moe_decoder.c names; ds_metal_is_available()
 * returns 0 so the reference always takes its CPU path.
 * Test infrastructure only. */
#include <stddef.h>
#include <stdint.h>
#include "ds_metal.h"
int ds_metal_is_available(const ds_metal_ctx_t *ctx) { (void)ctx; return 0; }
void ds_metal_moe_experts(ds_metal_ctx_t *ctx, const float *x, const uint16_t **gu,
                          const uint16_t **dn, const float *w, int k, int h, int i, float *o)
{ (void)ctx; (void)x; (void)gu; (void)dn; (void)w; (void)k; (void)h; (void)i; (void)o; }
void ds_metal_shared_experts(ds_metal_ctx_t *ctx, const float *x, const uint16_t *gu,
                             const uint16_t *dn, int h, int si, float *o)
{ (void)ctx; (void)x; (void)gu; (void)dn; (void)h; (void)si; (void)o; }
int ds_metal_lm_head_argmax(ds_metal_ctx_t *ctx, const float *x, const uint16_t *W, int h, int v)
{ (void)ctx; (void)x; (void)W; (void)h; (void)v; return -1; }
