/*
 * Minimal safetensors reader for the model loaders: mmaps every shard of a
 * transformer directory, indexes tensor names, and converts F32 / F16 / BF16
 * data to bf16 bits or f32 on the host for upload.  Reads the same files the
 * reference reads (iris_safetensors.c, safetensors_open :233;
 * open_transformer_shards iris_transformer_flux.c:473 — single file or the
 * shards named by diffusion_pytorch_model.safetensors.index.json).
 */
#include <fcntl.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include "iris_internal.h"

static const char *skip_ws(const char *p) {
    while (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t') p++;
    return p;
}

/* parse a JSON string starting at p (on the opening quote) into out */
static const char *parse_str(const char *p, char *out, size_t cap) {
    if (*p != '"') return NULL;
    p++;
    size_t n = 0;
    while (*p && *p != '"') {
        if (*p == '\\' && p[1]) p++;
        if (n + 1 < cap) out[n++] = *p;
        p++;
    }
    if (*p != '"') return NULL;
    out[n] = 0;
    return p + 1;
}

/* skip any JSON value */
static const char *skip_value(const char *p) {
    p = skip_ws(p);
    if (*p == '"') {
        char tmp[8];
        (void)tmp;
        p++;
        while (*p && *p != '"') {
            if (*p == '\\' && p[1]) p++;
            p++;
        }
        return *p ? p + 1 : p;
    }
    if (*p == '{' || *p == '[') {
        char open = *p, close = (*p == '{') ? '}' : ']';
        int depth = 0;
        do {
            if (*p == '"') {
                p = skip_value(p);
                continue;
            }
            if (*p == open) depth++;
            if (*p == close) depth--;
            p++;
        } while (*p && depth > 0);
        return p;
    }
    while (*p && *p != ',' && *p != '}' && *p != ']') p++;
    return p;
}

static int parse_header(st_model_t *m, int file, const char *hdr) {
    const char *p = skip_ws(hdr);
    if (*p != '{') return -1;
    p++;
    while (1) {
        p = skip_ws(p);
        if (*p == '}') break;
        char key[256];
        p = parse_str(p, key, sizeof(key));
        if (!p) return -1;
        p = skip_ws(p);
        if (*p != ':') return -1;
        p = skip_ws(p + 1);
        if (strcmp(key, "__metadata__") == 0) {
            p = skip_value(p);
        } else {
            if (*p != '{') return -1;
            st_tensor_t t;
            memset(&t, 0, sizeof(t));
            snprintf(t.name, sizeof(t.name), "%s", key);
            t.file = file;
            t.dtype = ST_OTHER;
            p++;
            size_t off0 = 0, off1 = 0;
            while (1) {
                p = skip_ws(p);
                if (*p == '}') { p++; break; }
                char f[64];
                p = parse_str(p, f, sizeof(f));
                if (!p) return -1;
                p = skip_ws(p);
                if (*p != ':') return -1;
                p = skip_ws(p + 1);
                if (strcmp(f, "dtype") == 0) {
                    char d[32];
                    p = parse_str(p, d, sizeof(d));
                    if (!p) return -1;
                    t.dtype = !strcmp(d, "F32") ? ST_F32 : !strcmp(d, "F16") ? ST_F16
                            : !strcmp(d, "BF16") ? ST_BF16 : !strcmp(d, "I8") ? ST_I8 : ST_OTHER;
                } else if (strcmp(f, "shape") == 0) {
                    if (*p != '[') return -1;
                    p++;
                    t.ndim = 0;
                    while (1) {
                        p = skip_ws(p);
                        if (*p == ']') { p++; break; }
                        char *end;
                        long long v = strtoll(p, &end, 10);
                        if (end == p) return -1;
                        if (t.ndim < 8) t.shape[t.ndim++] = v;
                        p = skip_ws(end);
                        if (*p == ',') p++;
                    }
                } else if (strcmp(f, "data_offsets") == 0) {
                    if (*p != '[') return -1;
                    char *end;
                    off0 = (size_t)strtoull(skip_ws(p + 1), &end, 10);
                    p = skip_ws(end);
                    if (*p == ',') p++;
                    off1 = (size_t)strtoull(skip_ws(p), &end, 10);
                    p = skip_ws(end);
                    if (*p != ']') return -1;
                    p++;
                } else {
                    p = skip_value(p);
                }
                p = skip_ws(p);
                if (*p == ',') p++;
            }
            t.offset = off0;
            t.nbytes = off1 - off0;
            st_tensor_t *nt = realloc(m->tensors, sizeof(st_tensor_t) * (m->ntensors + 1));
            if (!nt) return -1;
            m->tensors = nt;
            m->tensors[m->ntensors++] = t;
        }
        p = skip_ws(p);
        if (*p == ',') p++;
    }
    return 0;
}

static int open_file(st_model_t *m, const char *path) {
    if (m->nfiles >= 16) return -1;
    int fd = open(path, O_RDONLY);
    if (fd < 0) return -1;
    struct stat sb;
    if (fstat(fd, &sb) != 0 || sb.st_size < 8) { close(fd); return -1; }
    void *map = mmap(NULL, (size_t)sb.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    if (map == MAP_FAILED) { close(fd); return -1; }
    uint64_t hlen;
    memcpy(&hlen, map, 8);
    if (hlen + 8 > (uint64_t)sb.st_size) { munmap(map, (size_t)sb.st_size); close(fd); return -1; }
    char *hdr = malloc(hlen + 1);
    if (!hdr) { munmap(map, (size_t)sb.st_size); close(fd); return -1; }
    memcpy(hdr, (char *)map + 8, hlen);
    hdr[hlen] = 0;
    int f = m->nfiles;
    m->maps[f] = map;
    m->fds[f] = fd;
    m->sizes[f] = (size_t)sb.st_size;
    m->data_start[f] = 8 + hlen;
    m->nfiles++;
    int rc = parse_header(m, f, hdr);
    free(hdr);
    /* a tensor whose data runs past the end of the file (truncated download) fails the open */
    for (int i = 0; rc == 0 && i < m->ntensors; i++) {
        const st_tensor_t *t = &m->tensors[i];
        size_t avail = m->sizes[f] - m->data_start[f];  /* data_start <= size checked above */
        if (t->file == f && (t->offset > avail || t->nbytes > avail - t->offset))
            rc = -1;
    }
    return rc;
}

/* Opens the weights of a model directory: the shards named by a diffusers
 * (diffusion_pytorch_model.safetensors.index.json) or transformers
 * (model.safetensors.index.json, the text encoder's) index, else the single
 * diffusion_pytorch_model.safetensors or model.safetensors. */
int st_open_dir(st_model_t *m, const char *dir) {
    memset(m, 0, sizeof(*m));
    char path[4200];
    static const char *const index_names[2] = {"diffusion_pytorch_model.safetensors.index.json",
                                               "model.safetensors.index.json"};
    FILE *fp = NULL;
    for (int k = 0; k < 2 && !fp; k++) {
        snprintf(path, sizeof(path), "%s/%s", dir, index_names[k]);
        fp = fopen(path, "rb");
    }
    if (fp) {
        fseek(fp, 0, SEEK_END);
        long len = ftell(fp);
        fseek(fp, 0, SEEK_SET);
        char *js = malloc((size_t)len + 1);
        if (!js) { fclose(fp); return -1; }
        size_t got = fread(js, 1, (size_t)len, fp);
        fclose(fp);
        js[got] = 0;
        /* collect the distinct shard file names of "weight_map" values */
        char names[16][256];
        int nn = 0;
        const char *p = strstr(js, "\"weight_map\"");
        if (p) p = strchr(p, '{');
        while (p && *p && *p != '}') {
            p = strchr(p + 1, '"');  /* key */
            if (!p) break;
            char key[512];
            p = parse_str(p, key, sizeof(key));
            if (!p) break;
            p = strchr(p, '"');
            if (!p) break;
            char val[256];
            p = parse_str(p, val, sizeof(val));
            if (!p) break;
            int dup = 0;
            for (int i = 0; i < nn; i++) dup |= !strcmp(names[i], val);
            if (!dup && nn < 16) snprintf(names[nn++], 256, "%s", val);
            p = skip_ws(p);
        }
        free(js);
        for (int i = 0; i < nn; i++) {
            snprintf(path, sizeof(path), "%s/%s", dir, names[i]);
            if (open_file(m, path) != 0) { st_close(m); return -1; }
        }
        if (nn > 0) return 0;
    }
    snprintf(path, sizeof(path), "%s/diffusion_pytorch_model.safetensors", dir);
    FILE *single = fopen(path, "rb");
    if (!single) snprintf(path, sizeof(path), "%s/model.safetensors", dir);
    else fclose(single);
    if (open_file(m, path) != 0) { st_close(m); return -1; }
    return 0;
}

/* Opens one .safetensors file (a LoRA adapter, a single-file model). */
int st_open_file(st_model_t *m, const char *path) {
    memset(m, 0, sizeof(*m));
    if (open_file(m, path) != 0) { st_close(m); return -1; }
    return 0;
}

void st_close(st_model_t *m) {
    for (int i = 0; i < m->nfiles; i++) {
        munmap(m->maps[i], m->sizes[i]);
        close(m->fds[i]);
    }
    free(m->tensors);
    memset(m, 0, sizeof(*m));
}

const st_tensor_t *st_find(const st_model_t *m, const char *name) {
    for (int i = 0; i < m->ntensors; i++)
        if (strcmp(m->tensors[i].name, name) == 0) return &m->tensors[i];
    return NULL;
}

static size_t st_numel(const st_tensor_t *t) {
    size_t n = 1;
    for (int i = 0; i < t->ndim; i++) n *= (size_t)t->shape[i];
    return n;
}

static const uint8_t *st_data(const st_model_t *m, const st_tensor_t *t) {
    if (t->offset + t->nbytes + m->data_start[t->file] > m->sizes[t->file]) return NULL;
    return (const uint8_t *)m->maps[t->file] + m->data_start[t->file] + t->offset;
}

const void *st_raw(const st_model_t *m, const st_tensor_t *t) { return st_data(m, t); }

static float f16_to_f32(uint16_t h) {
    uint32_t s = (uint32_t)(h & 0x8000) << 16, e = (h >> 10) & 0x1F, f = h & 0x3FF, u;
    if (e == 0) {
        if (f == 0) u = s;
        else {
            e = 127 - 15 + 1;
            while (!(f & 0x400)) { f <<= 1; e--; }
            f &= 0x3FF;
            u = s | (e << 23) | (f << 13);
        }
    } else if (e == 31) u = s | 0x7F800000u | (f << 13);
    else u = s | ((e + 127 - 15) << 23) | (f << 13);
    union { uint32_t u; float f; } v = {u};
    return v.f;
}

int st_read_bf16(const st_model_t *m, const st_tensor_t *t, uint16_t *out, size_t numel) {
    if (t->dtype == ST_I8 || st_numel(t) != numel || t->nbytes != numel * (t->dtype == ST_F32 ? 4 : 2)) return -1;
    const uint8_t *d = st_data(m, t);
    if (!d) return -1;
    if (t->dtype == ST_BF16) { memcpy(out, d, numel * 2); return 0; }
    if (t->dtype == ST_F32) {
        const float *f = (const float *)d;
        for (size_t i = 0; i < numel; i++) out[i] = f32_to_bf16_bits(f[i]);
        return 0;
    }
    if (t->dtype == ST_F16) {
        const uint16_t *h = (const uint16_t *)d;
        for (size_t i = 0; i < numel; i++) out[i] = f32_to_bf16_bits(f16_to_f32(h[i]));
        return 0;
    }
    return -1;
}

int st_read_f32(const st_model_t *m, const st_tensor_t *t, float *out, size_t numel) {
    if (t->dtype == ST_I8 || st_numel(t) != numel || t->nbytes != numel * (t->dtype == ST_F32 ? 4 : 2)) return -1;
    const uint8_t *d = st_data(m, t);
    if (!d) return -1;
    if (t->dtype == ST_F32) { memcpy(out, d, numel * 4); return 0; }
    if (t->dtype == ST_BF16) {
        const uint16_t *b = (const uint16_t *)d;
        for (size_t i = 0; i < numel; i++) out[i] = bf16_bits_to_f32(b[i]);
        return 0;
    }
    if (t->dtype == ST_F16) {
        const uint16_t *h = (const uint16_t *)d;
        for (size_t i = 0; i < numel; i++) out[i] = f16_to_f32(h[i]);
        return 0;
    }
    return -1;
}

int json_get_number(const char *json, const char *key, double *out) {
    char pat[128];
    snprintf(pat, sizeof(pat), "\"%s\"", key);
    const char *p = strstr(json, pat);
    if (!p) return -1;
    p = strchr(p + strlen(pat), ':');
    if (!p) return -1;
    char *end;
    double v = strtod(p + 1, &end);
    if (end == p + 1) return -1;
    *out = v;
    return 0;
}
