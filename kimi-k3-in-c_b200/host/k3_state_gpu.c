/* k3_state_gpu.c -- the state file for device-resident state (include/k3_gpu.h).
 *
 * Same header as the reference's K3StateHdr (src/cli/k3_state.h:37-50) under version
 * K3G_STATE_VER; the payload is streamed between the device and the file through one
 * page-locked staging buffer, hashed on the way with FNV-1a folded eight bytes at a time
 * (offset basis and prime of FNV-1a; the reference's k3_state_hash, k3_state.c:47-62, uses
 * the same folding). Save publishes by rename after fsync, load checks every field it
 * sizes a read by before reading, then the length, then the hash (k3_state.c:102-183).
 */
#define _POSIX_C_SOURCE 200809L
#include "k3_gpu.h"

#include <errno.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/stat.h>
#include <unistd.h>

#include "k3_gpu_internal.h"

typedef struct {
    char magic[4];
    int32_t version;
    int32_t fp[12];
    int32_t n_bound, n_mla, cached, nseq;
    int64_t kper;
    int64_t kvpp, ropepp;
    uint64_t payload_hash;
} StateHdr;

#define HASH_INIT 0xcbf29ce484222325ULL
#define HASH_PRIME 0x100000001b3ULL
#define STAGE_BYTES ((size_t)64 << 20)

static uint64_t fold(uint64_t h, const void *p, size_t n)
{
    const unsigned char *b = (const unsigned char *)p;
    size_t i = 0;
    for (; i + 8 <= n; i += 8) {
        uint64_t w;
        memcpy(&w, b + i, 8);
        h = (h ^ w) * HASH_PRIME;
    }
    for (; i < n; i++) h = (h ^ b[i]) * HASH_PRIME;
    return h;
}

static uint64_t hdr_hash(const StateHdr *hd)
{
    StateHdr z = *hd;
    z.payload_hash = 0;
    return fold(HASH_INIT, &z, sizeof z);
}

static void *stage(void)
{
    static void *buf = NULL;
    if (!buf && k3cuda_host_alloc(k3g_ctx(), &buf, STAGE_BYTES) != K3CUDA_OK) {
        fprintf(stderr, "k3_state: cannot allocate the staging buffer: %s\n", k3cuda_last_error());
        buf = NULL;
    }
    return buf;
}

/* device -> file in staging-buffer pieces, hashed */
static int put_dev(FILE *f, const void *d, size_t bytes, uint64_t *h)
{
    char *st = (char *)stage();
    if (!st) return -1;
    for (size_t off = 0; off < bytes; off += STAGE_BYTES) {
        const size_t n = bytes - off < STAGE_BYTES ? bytes - off : STAGE_BYTES;
        if (k3cuda_memcpy_d2h(k3g_ctx(), st, (const char *)d + off, n) != K3CUDA_OK ||
            k3cuda_sync(k3g_ctx()) != K3CUDA_OK) {
            fprintf(stderr, "k3_state: device read failed: %s\n", k3cuda_last_error());
            return -1;
        }
        if (fwrite(st, 1, n, f) != n) return -1;
        *h = fold(*h, st, n);
    }
    return 0;
}

/* file -> device in staging-buffer pieces, hashed */
static int get_dev(FILE *f, void *d, size_t bytes, uint64_t *h)
{
    char *st = (char *)stage();
    if (!st) return -1;
    for (size_t off = 0; off < bytes; off += STAGE_BYTES) {
        const size_t n = bytes - off < STAGE_BYTES ? bytes - off : STAGE_BYTES;
        if (fread(st, 1, n, f) != n) return -1;
        *h = fold(*h, st, n);
        if (k3cuda_memcpy_h2d(k3g_ctx(), (char *)d + off, st, n) != K3CUDA_OK ||
            k3cuda_sync(k3g_ctx()) != K3CUDA_OK) {
            fprintf(stderr, "k3_state: device write failed: %s\n", k3cuda_last_error());
            return -1;
        }
    }
    return 0;
}

int k3g_state_save(const char *path, const int32_t fp[12], const int *seq, int nseq,
                   const float *d_ks, int64_t kper, int n_bound, const void *d_latent,
                   const void *d_rope, int n_mla, int kv_cap, int kv_lora, int rope_w,
                   int cached)
{
    if (nseq < 0 || cached < 0 || cached > nseq || cached > kv_cap || kper < 0 || n_bound < 0 ||
        n_mla < 0 || kv_lora < 0 || rope_w < 0) {
        fprintf(stderr, "k3_state: refusing to save inconsistent counts (nseq %d, cached %d, "
                        "cap %d)\n", nseq, cached, kv_cap);
        return -1;
    }
    char tmp[4096];
    if (snprintf(tmp, sizeof tmp, "%s.tmp.XXXXXX", path) >= (int)sizeof tmp) {
        fprintf(stderr, "%s: path too long\n", path);
        return -1;
    }
    const int fd = mkstemp(tmp);
    if (fd < 0) {
        fprintf(stderr, "cannot stage %s next to %s: %s\n", tmp, path, strerror(errno));
        return -1;
    }
    {
        const mode_t um = umask(0);
        umask(um);
        if (fchmod(fd, 0666 & ~um) != 0) {
            close(fd);
            unlink(tmp);
            return -1;
        }
    }
    FILE *f = fdopen(fd, "wb");
    if (!f) {
        close(fd);
        unlink(tmp);
        return -1;
    }
    StateHdr hd;
    memset(&hd, 0, sizeof hd);
    memcpy(hd.magic, "K3ST", 4);
    hd.version = K3G_STATE_VER;
    memcpy(hd.fp, fp, sizeof hd.fp);
    hd.n_bound = n_bound; hd.n_mla = n_mla; hd.cached = cached; hd.nseq = nseq;
    hd.kper = kper; hd.kvpp = kv_lora; hd.ropepp = rope_w;
    int rc = 0;
    uint64_t h = hdr_hash(&hd);
    if (fwrite(&hd, sizeof hd, 1, f) != 1) rc = -1;
    if (!rc && nseq && fwrite(seq, sizeof(int), (size_t)nseq, f) != (size_t)nseq) rc = -1;
    if (!rc) h = fold(h, seq, (size_t)nseq * sizeof(int));
    if (!rc) rc = put_dev(f, d_ks, (size_t)kper * n_bound * sizeof(float), &h);
    for (int m = 0; !rc && m < n_mla; m++)
        rc = put_dev(f, (const char *)d_latent + (size_t)m * kv_cap * kv_lora * 2,
                     (size_t)cached * kv_lora * 2, &h);
    for (int m = 0; !rc && m < n_mla; m++)
        rc = put_dev(f, (const char *)d_rope + (size_t)m * kv_cap * rope_w * 2,
                     (size_t)cached * rope_w * 2, &h);
    hd.payload_hash = h;
    if (!rc && fseek(f, 0, SEEK_SET) != 0) rc = -1;
    if (!rc && fwrite(&hd, sizeof hd, 1, f) != 1) rc = -1;
    if (!rc && fflush(f) != 0) rc = -1;
    if (!rc && fsync(fd) != 0) rc = -1;
    if (fclose(f) != 0) rc = -1;
    if (!rc && rename(tmp, path) != 0) rc = -1;
    if (rc) {
        fprintf(stderr, "failed writing %s: %s\n", path, strerror(errno));
        unlink(tmp);
    }
    return rc;
}

int k3g_state_load(const char *path, const int32_t fp[12], int *seq, int seq_cap, int *nseq,
                   float *d_ks, int64_t kper, int n_bound, void *d_latent, void *d_rope,
                   int n_mla, int kv_cap, int kv_lora, int rope_w, int *cached)
{
    FILE *f = fopen(path, "rb");
    if (!f) {
        perror(path);
        return -1;
    }
    StateHdr hd;
    if (fread(&hd, sizeof hd, 1, f) != 1 || memcmp(hd.magic, "K3ST", 4) != 0) {
        fprintf(stderr, "%s is not a k3 state file\n", path);
        fclose(f);
        return -1;
    }
    const char *why = NULL;
    if (hd.version != K3G_STATE_VER) why = "a state version this build does not read";
    else if (memcmp(hd.fp, fp, sizeof hd.fp) != 0) why = "state of a different model architecture";
    else if (hd.n_bound != n_bound || hd.n_mla != n_mla) why = "a different number of layers";
    else if (hd.kper != kper || hd.kvpp != kv_lora || hd.ropepp != rope_w)
        why = "a different per-layer state geometry";
    else if (hd.nseq < 0 || hd.cached < 0 || hd.cached > hd.nseq) why = "inconsistent counts";
    else if (hd.nseq > seq_cap) why = "more token ids than the caller's buffer holds";
    else if (hd.cached > kv_cap) why = "more positions than this run's cache holds";
    if (why) {
        fprintf(stderr, "REFUSING: %s holds %s (version %d)\n", path, why, hd.version);
        fclose(f);
        return -1;
    }
    int rc = 0;
    uint64_t h = hdr_hash(&hd);
    if (hd.nseq && fread(seq, sizeof(int), (size_t)hd.nseq, f) != (size_t)hd.nseq) rc = -1;
    if (!rc) h = fold(h, seq, (size_t)hd.nseq * sizeof(int));
    if (!rc) rc = get_dev(f, d_ks, (size_t)kper * n_bound * sizeof(float), &h);
    for (int m = 0; !rc && m < n_mla; m++)
        rc = get_dev(f, (char *)d_latent + (size_t)m * kv_cap * kv_lora * 2,
                     (size_t)hd.cached * kv_lora * 2, &h);
    for (int m = 0; !rc && m < n_mla; m++)
        rc = get_dev(f, (char *)d_rope + (size_t)m * kv_cap * rope_w * 2,
                     (size_t)hd.cached * rope_w * 2, &h);
    const int trailing = !rc && fgetc(f) != EOF;
    fclose(f);
    if (rc) {
        fprintf(stderr, "%s is truncated\n", path);
        return -1;
    }
    if (trailing) {
        fprintf(stderr, "REFUSING: %s is longer than its header describes\n", path);
        return -1;
    }
    if (h != hd.payload_hash) {
        fprintf(stderr, "REFUSING: %s does not hash to what its header says (header %016llx, "
                        "contents %016llx)\n", path, (unsigned long long)hd.payload_hash,
                (unsigned long long)h);
        return -1;
    }
    *nseq = hd.nseq;
    *cached = hd.cached;
    return 0;
}
