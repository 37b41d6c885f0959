/* vqprof_ref.c — test infrastructure: a command-line driver over the reference's own
 * tools/vq/gpu/vq-profile.h (included from the reference tree where it lies, never copied),
 * so the golden vectors of tests/golden/vqprof/ come from the reference's fingerprint and
 * reader themselves.
 *
 *   vqprof_ref fp DIR      the artifact fingerprint (vqprof_artifact), 16 hex digits
 *   vqprof_ref load PATH   vqprof_load's return code, header fields and entries, one per line
 */
#include <stdio.h>
#include <string.h>

#include "vq-profile.h"

int main(int argc, char **argv) {
    if (argc == 3 && !strcmp(argv[1], "fp")) {
        unsigned long long fp = 0;
        const int rc = vqprof_artifact(argv[2], &fp);
        printf("%d %016llx\n", rc, fp);
        return 0;
    }
    if (argc == 3 && !strcmp(argv[1], "load")) {
        static vqprof pf;
        const int rc = vqprof_load(argv[2], &pf);
        printf("rc %d\nartifact %016llx\ngpu %s\ndriver %s\nn %d\n", rc, pf.artifact, pf.gpu, pf.driver, pf.n);
        for (int i = 0; i < pf.n; i++) {
            const vqprof_entry *e = &pf.e[i];
            printf("entry %d %d %d %d %d %d %d %d %d %d\n", e->kind, e->dim, e->nc, e->rows, e->cols, e->v3, e->variant,
                   e->threads, e->bn, e->bk);
        }
        return 0;
    }
    fprintf(stderr, "usage: vqprof_ref fp DIR | load PATH\n");
    return 2;
}
