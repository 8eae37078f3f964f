/* The C ABI from plain C, as a Rust (or any FFI) binding would use it: the header compiles as C,
 * the library links, and the entry points that need no GPU answer: the ABI version, the placement
 * words of a batch (crates/graph/src/decode.rs:1073-1092), the sampler's schedule and Euler steps
 * (crates/graph/src/local/dit.rs:39-81), and a context that fails loudly without an sm_100 GPU. */
#include <stdio.h>
#include <string.h>

#include "tgcuda.h"

int main(void) {
    if (tg_abi_version() != TGCUDA_ABI_VERSION) return 1;
    /* Batch::placement: rows (5, slot 0), spare, (2, slot 2) over 3 slots. */
    tg_row rows[3] = {{5, 0}, {TG_SPARE, 0}, {2, 2}};
    uint32_t words[6], n = 0;
    if (tg_batch_placement(3, 3, rows, 16, words, &n) != TG_OK || n != 6) return 2;
    const uint32_t want[6] = {5, TG_SPARE, 2, 0, TG_SPARE, 2};
    for (int i = 0; i < 6; i++)
        if (words[i] != want[i]) return 3;
    /* Two rows in one slot are refused, with a message. */
    tg_row twice[2] = {{1, 1}, {2, 1}};
    if (tg_batch_placement(2, 2, twice, 16, words, &n) != TG_ESHAPE || strlen(tg_last_error()) == 0) return 4;
    float sched[11];
    if (tg_cfm_schedule(10, sched) != TG_OK || sched[10] != 0.0f || !(sched[0] > 0.999f)) return 5;
    float t[16], dt[16];
    size_t count = 0;
    if (tg_cfm_euler_steps(10, t, dt, 16, &count) != TG_OK || count != 9) return 6;
    tg_ctx *ctx = NULL;
    const int st = tg_ctx_create(0, &ctx);
    printf("ctx %d (%s)\n", st, tg_last_error());
    if (st == TG_OK) tg_ctx_destroy(ctx);
    else if (st != TG_ENODEVICE || ctx != NULL) return 7;
    printf("ok\n");
    return 0;
}
