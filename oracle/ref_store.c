/* ref_store.c - the reference's own expert store driven by a scripted trace,
 * to replay the same trace through libtlmg's slot policy (tlmg_store_*).
 *
 * TEST INFRASTRUCTURE ONLY. The reference's src/lib/tlm_store.c is compiled
 * in place through the #include below (nothing is copied), so the driver can
 * wait until no load is in flight (quiesce) and read each slot's state: the
 * replay is then deterministic (a load completes exactly where the trace
 * says so, not when the disk answers). The store is opened over a manifest
 * made by the reference's tlmc, as tierlm opens it, with n_slots slots.
 */
#define _GNU_SOURCE 1
#include "tlm_store.c"

#include "tlm_io.h"

typedef struct {
    tlm_manifest m;
    tlm_io *io;
    tlm_store *st;
    tlm_expert_ref refs[1024];
    int n_refs;
} refstore;

void refstore_close(void *p) {
    refstore *R = (refstore *)p;
    if (!R) return;
    for (int i = 0; i < R->n_refs; i++) tlm_store_release(R->st, &R->refs[i]);
    if (R->st) tlm_store_close(R->st);
    if (R->io) tlm_io_close(R->io);
    tlm_manifest_free(&R->m);
    free(R);
}

void *refstore_open(const char *manifest, int n_slots) {
    refstore *R = (refstore *)calloc(1, sizeof *R);
    if (!R || tlm_manifest_load(&R->m, manifest)) { free(R); return NULL; }
    char paths[TLM_MAX_DRIVES][1024];
    const char *pp[TLM_MAX_DRIVES];
    for (uint32_t d = 0; d < R->m.n_drives; d++) {
        tlm_manifest_drive_path(&R->m, (int)d, paths[d], sizeof paths[d]);
        pp[d] = paths[d];
    }
    tlm_io_opts io;
    memset(&io, 0, sizeof io);
    io.backend = TLM_IO_PREAD;
    io.threads_per_drive = 4;
    io.queue_depth = 32;
    R->io = tlm_io_open(pp, (int)R->m.n_drives, &io);
    if (!R->io) { refstore_close(R); return NULL; }
    uint64_t slot = 0;
    for (uint32_t i = 0; i < R->m.n_packets; i++)
        if (R->m.packets[i].type == TLM_PK_EXPERT && R->m.packets[i].total_len > slot) slot = R->m.packets[i].total_len;
    tlm_store_opts so;
    memset(&so, 0, sizeof so);
    so.budget_bytes = (uint64_t)n_slots * slot;
    so.prefetch = 1;
    R->st = tlm_store_open(&R->m, R->io, &so);
    if (!R->st) { refstore_close(R); return NULL; }
    return R;
}

/* demand acquisition (refs kept until refstore_wait_release) */
int refstore_acquire(void *p, int layer, const int *ids, int k) {
    refstore *R = (refstore *)p;
    int rc = tlm_store_acquire(R->st, layer, ids, k, R->refs + R->n_refs);
    R->n_refs += k;
    return rc;
}

void refstore_prefetch(void *p, int layer, const int *ids, int k) {
    tlm_store_prefetch(((refstore *)p)->st, layer, ids, k);
}

/* every load in flight completes */
void refstore_quiesce(void *p) {
    tlm_store *s = ((refstore *)p)->st;
    pthread_mutex_lock(&s->mu);
    while (s->loading > 0) pthread_cond_wait(&s->cv, &s->mu);
    pthread_mutex_unlock(&s->mu);
}

/* wait for every held reference (as moe() does), quiesce, release them */
int refstore_wait_release(void *p) {
    refstore *R = (refstore *)p;
    int rc = 0;
    for (int i = 0; i < R->n_refs; i++)
        if (R->refs[i].slot >= 0 && tlm_store_wait(R->st, &R->refs[i]) && !rc) rc = -1;
    refstore_quiesce(p);
    for (int i = 0; i < R->n_refs; i++) tlm_store_release(R->st, &R->refs[i]);
    R->n_refs = 0;
    return rc;
}

void refstore_tick(void *p) { tlm_store_tick(((refstore *)p)->st); }

int refstore_n_slots(void *p) { return ((refstore *)p)->st->n_slots; }

/* slot state: state, key (layer * n_experts + id, -1 = none), refcount, prefetched */
void refstore_slot(void *p, int i, int *out) {
    tlm_store *s = ((refstore *)p)->st;
    pthread_mutex_lock(&s->mu);
    const st_slot *sl = &s->slots[i];
    out[0] = sl->state;
    out[1] = sl->ex >= 0 ? (int)(s->ex[sl->ex].loc.layer * s->geom.n_experts + s->ex[sl->ex].loc.id) : -1;
    out[2] = sl->refcount;
    out[3] = sl->prefetched;
    pthread_mutex_unlock(&s->mu);
}

/* hits, misses, prefetch issued, prefetch used, prefetch dropped, evictions */
void refstore_stats(void *p, int64_t *out) {
    tlm_store_stats st;
    tlm_store_get_stats(((refstore *)p)->st, &st);
    out[0] = (int64_t)st.hits;
    out[1] = (int64_t)st.misses;
    out[2] = (int64_t)st.prefetch_issued;
    out[3] = (int64_t)st.prefetch_used;
    out[4] = (int64_t)st.prefetch_dropped;
    out[5] = (int64_t)st.evictions;
}
