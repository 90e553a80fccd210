/* CPU restatement of the capacity-ceiling routing rule -- TEST INFRASTRUCTURE ONLY.
 *
 * Used by tests/ and by bench.py's CPU-baseline leg as the checker and the
 * timed CPU port; the product library never links it.
 *
 * Follows Router::assign_effective_experts, src/orchestration/router.hpp:249-266
 * (independently restated by the reference at tests/test_orchestration.cpp:187-205):
 * tokens are grouped by primary expert, each group ranked by batch_position;
 * rank < capacity keeps the primary, later ones take their own secondary.
 * One hop only -- the secondary is not capacity-checked (router.hpp:21-27).
 */
#include <stdint.h>
#include <stdlib.h>

typedef struct {
    uint32_t primary;
    uint32_t position;
    uint64_t index;
} unit_key;

static int cmp_unit(const void* a, const void* b) {
    const unit_key* x = (const unit_key*)a;
    const unit_key* y = (const unit_key*)b;
    if (x->primary != y->primary) return x->primary < y->primary ? -1 : 1;
    if (x->position != y->position) return x->position < y->position ? -1 : 1;
    return x->index < y->index ? -1 : (x->index > y->index);
}

/* effective[i] for n tokens.  capacity == UINT64_MAX means unlimited
 * (RouterConfig default, router.hpp:50).  Returns 0, or -1 on allocation failure. */
int oracle_capacity_assign(const uint32_t* primary, const uint32_t* secondary,
                           const uint32_t* batch_position, uint64_t n,
                           uint64_t capacity, uint32_t* effective) {
    if (n == 0) return 0;
    unit_key* keys = (unit_key*)malloc(sizeof(unit_key) * n);
    if (!keys) return -1;
    for (uint64_t i = 0; i < n; ++i) {
        keys[i].primary = primary[i];
        keys[i].position = batch_position[i];
        keys[i].index = i;
    }
    qsort(keys, n, sizeof(unit_key), cmp_unit);
    uint64_t rank = 0;
    for (uint64_t i = 0; i < n; ++i) {
        if (i > 0 && keys[i].primary != keys[i - 1].primary) rank = 0;
        uint64_t src = keys[i].index;
        effective[src] = rank < capacity ? primary[src] : secondary[src];
        ++rank;
    }
    free(keys);
    return 0;
}

/* Slot-major MoE units from the gating indices idx_ext[T][ldi] (k chosen
 * experts followed by the (k+1)-th choice when k < E): unit u = j*T + t has
 * batch_position u, primary idx[t][j], secondary idx[t][k] (or the primary
 * when k == E).  Writes effective[T*k]. */
int oracle_moe_route(const int32_t* idx_ext, uint64_t T, uint32_t ldi, uint32_t k,
                     uint32_t num_experts, uint64_t capacity, uint32_t* effective) {
    uint64_t n = T * (uint64_t)k;
    if (n == 0) return 0;
    uint32_t* p = (uint32_t*)malloc(sizeof(uint32_t) * n * 3);
    if (!p) return -1;
    uint32_t* s = p + n;
    uint32_t* pos = s + n;
    for (uint32_t j = 0; j < k; ++j)
        for (uint64_t t = 0; t < T; ++t) {
            uint64_t u = j * T + t;
            p[u] = (uint32_t)idx_ext[t * ldi + j];
            s[u] = k < num_experts ? (uint32_t)idx_ext[t * ldi + k] : p[u];
            pos[u] = (uint32_t)u;
        }
    int rc = oracle_capacity_assign(p, s, pos, n, capacity, effective);
    free(p);
    return rc;
}
