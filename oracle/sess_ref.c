/* Reference session KV file calls (test infrastructure, reference build only).
 *
 * Wraps the reference's own sess_kv_save / sess_kv_load (cache.c:174-195,
 * 219-247), compiled from the reference tree, around a zeroed Engine that
 * carries only what those two functions read: the header's n_blocks, the KV
 * blob, kv_dim and max_seq (yllm.h:107-111). */
#include <stdint.h>
#include <stdlib.h>

#include "yllm.h"

int sess_kv_save(Engine* e, uint32_t pos, const char* path);
int sess_kv_load(Engine* e, const char* path, uint32_t* pos);

static Engine* engine_of(uint16_t* kv, uint32_t nb, uint32_t kv_dim, uint32_t max_seq)
{
    Engine* e = (Engine*)calloc(1, sizeof(Engine));
    if (!e) return NULL;
    e->ws.model.h.n_blocks = nb;
    e->kv = kv;
    e->kv_dim = kv_dim;
    e->max_seq = max_seq;
    return e;
}

int orc_sess_kv_save(const uint16_t* kv, uint32_t nb, uint32_t kv_dim, uint32_t max_seq, uint32_t pos,
                     const char* path)
{
    Engine* e = engine_of((uint16_t*)kv, nb, kv_dim, max_seq);
    int rc = e ? sess_kv_save(e, pos, path) : -1;
    free(e);
    return rc;
}

int orc_sess_kv_load(uint16_t* kv, uint32_t nb, uint32_t kv_dim, uint32_t max_seq, const char* path, uint32_t* pos)
{
    Engine* e = engine_of(kv, nb, kv_dim, max_seq);
    int rc = e ? sess_kv_load(e, path, pos) : -1;
    free(e);
    return rc;
}
