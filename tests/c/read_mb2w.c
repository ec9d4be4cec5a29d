/* Lists an MB2W file with include/mb2w_file.h: the meta records, then one
 * line per tensor (name dtype ndim shape offset nbytes scheme group in_dim) and
 * an FNV-1a hash of its bytes.  Used by tests/test_export.py. */
#include <stdio.h>
#include <stdlib.h>

#include "../../include/mb2w_file.h"

int main(int argc, char **argv) {
    if (argc != 2) return 2;
    FILE *f = fopen(argv[1], "rb");
    if (!f) return 3;
    fseek(f, 0, SEEK_END);
    long size = ftell(f);
    fseek(f, 0, SEEK_SET);
    unsigned char *buf = (unsigned char *)malloc((size_t)size);
    if (!buf || fread(buf, 1, (size_t)size, f) != (size_t)size) return 4;
    fclose(f);
    const mb2w_header *h;
    const mb2w_meta *m;
    const mb2w_tensor *t;
    int rc = mb2w_parse(buf, (size_t)size, &h, &m, &t);
    if (rc) {
        printf("error %d\n", rc);
        return 0;
    }
    printf("d_model %lld\n", (long long)mb2w_meta_get(h, m, "d_model", -1));
    printf("n_layers %lld\n", (long long)mb2w_meta_get(h, m, "n_layers", -1));
    for (uint32_t i = 0; i < h->n_tensors; ++i) {
        uint64_t hash = 1469598103934665603ull;
        for (uint64_t j = 0; j < t[i].nbytes; ++j) {
            hash ^= buf[t[i].offset + j];
            hash *= 1099511628211ull;
        }
        printf("%s %u %u %lld %lld %lld %lld %llu %llu %d %d %lld %016llx\n", t[i].name,
               t[i].dtype, t[i].ndim, (long long)t[i].shape[0], (long long)t[i].shape[1],
               (long long)t[i].shape[2], (long long)t[i].shape[3],
               (unsigned long long)t[i].offset, (unsigned long long)t[i].nbytes, t[i].scheme,
               t[i].group_size, (long long)t[i].in_dim, (unsigned long long)hash);
    }
    const mb2w_tensor *a = mb2w_find(h, t, "A_log");
    if (!a) a = mb2w_find(h, t, "layers.0.mixer.A_log");
    printf("found_A_log %d\n", a != NULL);
    free(buf);
    return 0;
}
