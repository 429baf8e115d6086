/*
 * TEST INFRASTRUCTURE ONLY -- the parity oracle, never the product.
 *
 * CPU float64 restatement of the reference MACE MH1 evaluation (LipidL/LASP-PIS):
 *   - neighbour semantics: lapis/src/runtime.cu:80-203 (cell validation, H^-1, plane
 *     heights, images, grid, wrap + winding) and lapis/include/lapis/pair.cuh:58-62,131
 *     (float32 displacement, inclusive cutoff, all images, (i,i,0) excluded);
 *   - model: mace/src/mh1.cu:107-235 (node kernels), 246-470 (pair forward/backward),
 *     471-537 (ZBL), 754-898 (stage order, scale/shift, e0 on the host) and
 *     mace/src/mh1_math.cuh (envelope, harmonics, radial MLP with LayerNorm + SiLU);
 *   - archive: mace/src/mh1.cu:626-734 (PWMH1001 records and their validation).
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load this file's
 * library.  Node tensors here are node-major: per node, every irrep block stores
 * [component][channel] at the block's e3nn offset.
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define NB 10
#define HID 64
#define CH 128

typedef struct {
  char *name;
  uint64_t size;
  unsigned char *data;
} Rec;
typedef struct {
  int in_off, out_off, in_mul, out_mul, dim, w_off;
} Path;
typedef struct {
  int in, out, np;
  const Path *p;
  const float *w;
} Lin;
typedef struct {
  const float *source, *target, *radial, *b0, *W[3], *bias[3], *gamma[3], *beta[3], *ow, *ob;
  int depth, outputs;
} Rad;
typedef struct {
  int path, in, sh, out;
} Term;
typedef struct {
  int out, deg, a, b, c;
} Poly;
typedef struct {
  Lin up, res, one, two, skip, plin;
  Rad radial, density;
  double alpha, beta;
  int nterms, paths, in_comp, out_comp;
  const Term *tp;
  const float *cg;
  int npoly, pouts;
  const Poly *poly;
  const float *pcoef;
} Layer;
typedef struct {
  Rec *recs;
  int nrec;
  float c[14];
  int species, lookup[119];
  float e0[119];
  const float *emb, *bessel, *radii, *zradii, *zc;
  Layer L[2];
  Lin read0, read1up, read1down;
} Model;

static void seterr(char *err, int cap, const char *msg) {
  if (err && cap > 0) {
    strncpy(err, msg, (size_t)cap - 1);
    err[cap - 1] = 0;
  }
}

/* ---------------- archive ---------------- */
static const Rec *find(const Model *m, const char *name) {
  for (int k = 0; k < m->nrec; ++k)
    if (!strcmp(m->recs[k].name, name))
      return &m->recs[k];
  return NULL;
}
static const float *fl(const Model *m, const char *name, uint64_t count, const char **bad) {
  const Rec *r = find(m, name);
  if (!r || (count && r->size != count * 4)) {
    if (!*bad)
      *bad = name;
    return NULL;
  }
  return (const float *)r->data;
}
static int get_linear(Model *m, const char *key, int in, int out, Lin *l, const char **bad) {
  char name[256];
  snprintf(name, sizeof name, "%s.dims", key);
  const Rec *d = find(m, name);
  if (!d || d->size != 8 || ((int *)d->data)[0] != in || ((int *)d->data)[1] != out) {
    *bad = "linear dims";
    return -1;
  }
  snprintf(name, sizeof name, "%s.paths", key);
  const Rec *p = find(m, name);
  snprintf(name, sizeof name, "%s.weight", key);
  const Rec *w = find(m, name);
  if (!p || !w || p->size % 24) {
    *bad = "linear records";
    return -1;
  }
  l->in = in;
  l->out = out;
  l->np = (int)(p->size / 24);
  l->p = (const Path *)p->data;
  l->w = (const float *)w->data;
  for (int k = 0; k < l->np; ++k) {
    Path q = l->p[k];
    if (q.in_mul <= 0 || q.out_mul <= 0 || q.dim < 1 || q.dim > 7 || q.in_off < 0 || q.out_off < 0 ||
        (int64_t)q.in_off + (int64_t)q.in_mul * q.dim > in ||
        (int64_t)q.out_off + (int64_t)q.out_mul * q.dim > out ||
        (uint64_t)q.w_off + (uint64_t)q.in_mul * q.out_mul > w->size / 4) {
      *bad = "linear path";
      return -1;
    }
  }
  return 0;
}
static void get_radial(Model *m, const char *key, int depth, int outputs, Rad *r, const char **bad) {
  char name[256];
  int s = m->species;
  snprintf(name, sizeof name, "%s.source", key);
  r->source = fl(m, name, (uint64_t)s * 64, bad);
  snprintf(name, sizeof name, "%s.target", key);
  r->target = fl(m, name, (uint64_t)s * 64, bad);
  snprintf(name, sizeof name, "%s.radial", key);
  r->radial = fl(m, name, 640, bad);
  snprintf(name, sizeof name, "%s.0.bias", key);
  r->b0 = fl(m, name, 64, bad);
  for (int k = 0; k < depth; ++k) {
    snprintf(name, sizeof name, "%s.%d.weight", key, 3 * k);
    r->W[k] = fl(m, name, k ? 64 * 64 : 64 * 1034, bad);
    snprintf(name, sizeof name, "%s.%d.bias", key, 3 * k);
    r->bias[k] = fl(m, name, 64, bad);
    snprintf(name, sizeof name, "%s.%d.weight", key, 3 * k + 1);
    r->gamma[k] = fl(m, name, 64, bad);
    snprintf(name, sizeof name, "%s.%d.bias", key, 3 * k + 1);
    r->beta[k] = fl(m, name, 64, bad);
  }
  snprintf(name, sizeof name, "%s.%d.weight", key, 3 * depth);
  r->ow = fl(m, name, (uint64_t)outputs * 64, bad);
  snprintf(name, sizeof name, "%s.%d.bias", key, 3 * depth);
  r->ob = fl(m, name, (uint64_t)outputs, bad);
  r->depth = depth;
  r->outputs = outputs;
}

void oracle_free(void *h) {
  Model *m = (Model *)h;
  if (!m)
    return;
  for (int k = 0; k < m->nrec; ++k) {
    free(m->recs[k].name);
    free(m->recs[k].data);
  }
  free(m->recs);
  free(m);
}

static int ends_with(const char *s, const char *t) {
  size_t a = strlen(s), b = strlen(t);
  return a >= b && !strcmp(s + a - b, t);
}

void *oracle_load(const char *path, char *err, int errcap) {
  FILE *f = fopen(path, "rb");
  if (!f) {
    seterr(err, errcap, "Cannot open MH1 archive");
    return NULL;
  }
  Model *m = (Model *)calloc(1, sizeof(Model));
  const char *bad = NULL;
  char magic[8];
  uint32_t count = 0;
  if (fread(magic, 1, 8, f) != 8 || memcmp(magic, "PWMH1001", 8)) {
    bad = "Invalid MH1 archive magic";
    goto fail;
  }
  if (fread(&count, 4, 1, f) != 1 || count == 0 || count > 10000) {
    bad = "Invalid MH1 tensor count";
    goto fail;
  }
  m->recs = (Rec *)calloc(count, sizeof(Rec));
  for (uint32_t k = 0; k < count; ++k) {
    uint32_t len = 0;
    uint64_t size = 0;
    if (fread(&len, 4, 1, f) != 1 || fread(&size, 8, 1, f) != 1 || !len || len > 1024 ||
        size > 512ull * 1024 * 1024 || size % 4) {
      bad = "Invalid MH1 archive record";
      goto fail;
    }
    Rec *r = &m->recs[m->nrec];
    r->name = (char *)calloc(len + 1, 1);
    r->data = (unsigned char *)malloc(size ? size : 1);
    r->size = size;
    m->nrec++;
    if (fread(r->name, 1, len, f) != len || (size && fread(r->data, 1, size, f) != size)) {
      bad = "Truncated MH1 archive";
      goto fail;
    }
    for (int q = 0; q + 1 < m->nrec; ++q)
      if (!strcmp(m->recs[q].name, r->name)) {
        bad = "Duplicate MH1 tensor";
        goto fail;
      }
    int indices = !strcmp(r->name, "atomic_numbers") || ends_with(r->name, ".dims") ||
                  ends_with(r->name, ".paths") || ends_with(r->name, ".terms");
    if (!indices)
      for (uint64_t q = 0; q < size / 4; ++q)
        if (!isfinite(((float *)r->data)[q])) {
          bad = "Nonfinite MH1 tensor";
          goto fail;
        }
  }
  fclose(f);
  f = NULL;
  {
    const float *c = fl(m, "constants", 14, &bad);
    if (!c || c[0] != 6) {
      bad = "Unsupported MH1 constants";
      goto fail;
    }
    memcpy(m->c, c, sizeof m->c);
    const Rec *zs = find(m, "atomic_numbers");
    if (!zs) {
      bad = "Missing atomic_numbers";
      goto fail;
    }
    m->species = (int)(zs->size / 4);
    if (m->species < 1 || m->species > 118) {
      bad = "Invalid MH1 element count";
      goto fail;
    }
    m->emb = fl(m, "embedding", (uint64_t)m->species * 512, &bad);
    m->bessel = fl(m, "bessel", 10, &bad);
    m->radii = fl(m, "radii", 119, &bad);
    m->zradii = fl(m, "zbl.radii", 119, &bad);
    m->zc = fl(m, "zbl.c", 4, &bad);
    const float *e0 = fl(m, "e0", (uint64_t)m->species, &bad);
    if (bad)
      goto fail;
    for (int z = 0; z < 119; ++z)
      m->lookup[z] = -1;
    for (int k = 0; k < m->species; ++k) {
      int z = ((const int *)zs->data)[k];
      if (z < 1 || z > 118 || m->lookup[z] >= 0) {
        bad = "Invalid MH1 element map";
        goto fail;
      }
      m->lookup[z] = k;
      m->e0[z] = e0[k];
    }
    for (int k = 0; k < 2; ++k) {
      Layer *l = &m->L[k];
      char p[64], name[256];
      snprintf(p, sizeof p, "layer%d", k);
#define LIN(field, key, i, o)                                                                      \
  snprintf(name, sizeof name, "%s.%s", p, key);                                                    \
  if (get_linear(m, name, i, o, &l->field, &bad))                                                 \
    goto fail;
      LIN(up, "linear_up", k ? 2048 : 512, k ? 512 : 128)
      LIN(res, "linear_res", k ? 512 : 128, 9728)
      LIN(one, "linear_1", k ? 5120 : 2048, 9728)
      LIN(two, "linear_2", 8192, 8192)
      LIN(skip, "skip_tp", k ? 2048 : 512, k ? 512 : 2048)
      LIN(plin, "product.linear", k ? 512 : 2048, k ? 512 : 2048)
#undef LIN
      snprintf(name, sizeof name, "%s.norm", p);
      const float *norm = fl(m, name, 2, &bad);
      snprintf(name, sizeof name, "%s.tp.dims", p);
      const Rec *dims = find(m, name);
      snprintf(name, sizeof name, "%s.tp.terms", p);
      const Rec *terms = find(m, name);
      snprintf(name, sizeof name, "%s.tp.values", p);
      const Rec *values = find(m, name);
      if (bad || !dims || dims->size != 12 || !terms || !values ||
          terms->size != values->size * 4) {
        bad = bad ? bad : "tensor product records";
        goto fail;
      }
      l->alpha = norm[0];
      l->beta = norm[1];
      l->paths = ((int *)dims->data)[0];
      l->in_comp = ((int *)dims->data)[1];
      l->out_comp = ((int *)dims->data)[2];
      if (l->paths != (k ? 10 : 4) || l->in_comp != (k ? 4 : 1) || l->out_comp != (k ? 40 : 16)) {
        bad = "Unsupported MH1 tensor product shape";
        goto fail;
      }
      l->nterms = (int)(values->size / 4);
      l->tp = (const Term *)terms->data;
      l->cg = (const float *)values->data;
      for (int t = 0; t < l->nterms; ++t) {
        Term q = l->tp[t];
        if (q.path < 0 || q.path >= l->paths || q.in < 0 || q.in >= l->in_comp || q.sh < 0 ||
            q.sh >= 16 || q.out < 0 || q.out >= l->out_comp) {
          bad = "Invalid MH1 tensor-product index";
          goto fail;
        }
      }
      snprintf(name, sizeof name, "%s.radial", p);
      get_radial(m, name, 3, l->paths * CH, &l->radial, &bad);
      snprintf(name, sizeof name, "%s.density", p);
      get_radial(m, name, 1, 1, &l->density, &bad);
      snprintf(name, sizeof name, "%s.product.terms", p);
      const Rec *pt = find(m, name);
      if (bad || !pt || pt->size % 20) {
        bad = bad ? bad : "product terms";
        goto fail;
      }
      l->npoly = (int)(pt->size / 20);
      l->poly = (const Poly *)pt->data;
      l->pouts = k ? 1 : 4;
      snprintf(name, sizeof name, "%s.product.coefficients", p);
      l->pcoef = fl(m, name, (uint64_t)l->npoly * 512, &bad);
      if (bad)
        goto fail;
      for (int t = 0; t < l->npoly; ++t) {
        Poly q = l->poly[t];
        if (q.deg < 1 || q.deg > 3 || q.out < 0 || q.out >= l->pouts || q.a < 0 || q.a >= 16 ||
            (q.deg >= 2 && (q.b < 0 || q.b >= 16)) || (q.deg == 3 && (q.c < 0 || q.c >= 16))) {
          bad = "Invalid MH1 polynomial index";
          goto fail;
        }
      }
    }
    if (get_linear(m, "readout0", 2048, 1, &m->read0, &bad) ||
        get_linear(m, "readout1.up", 512, 16, &m->read1up, &bad) ||
        get_linear(m, "readout1.down", 16, 1, &m->read1down, &bad))
      goto fail;
  }
  return m;
fail:
  if (f)
    fclose(f);
  seterr(err, errcap, bad ? bad : "Invalid MH1 archive");
  oracle_free(m);
  return NULL;
}

/* ---------------- neighbours (lapis semantics) ---------------- */
typedef struct {
  int i, j, s[3];
  float d[3];
} Edge;

typedef struct {
  double h[9], inv[9];
  int dims[3], images[3], grid_ok;
} Geometry;

static int geometry(const float *cell, float cutoff, int n, Geometry *g, char *err, int cap) {
  double *h = g->h;
  for (int k = 0; k < 9; ++k) {
    h[k] = cell[k];
    if (!isfinite(h[k])) {
      seterr(err, cap, "Nonfinite cell");
      return -1;
    }
  }
  double det = h[0] * (h[4] * h[8] - h[5] * h[7]) - h[1] * (h[3] * h[8] - h[5] * h[6]) +
               h[2] * (h[3] * h[7] - h[4] * h[6]);
  double scale = 0;
  for (int k = 0; k < 9; ++k)
    scale = fmax(scale, fabs(h[k]));
  if (!isfinite(det) || scale == 0 || fabs(det) < 1e-10 * scale * scale * scale) {
    seterr(err, cap, "Singular or ill-conditioned cell");
    return -1;
  }
  double *inv = g->inv;
  inv[0] = (h[4] * h[8] - h[5] * h[7]) / det;
  inv[1] = (h[2] * h[7] - h[1] * h[8]) / det;
  inv[2] = (h[1] * h[5] - h[2] * h[4]) / det;
  inv[3] = (h[5] * h[6] - h[3] * h[8]) / det;
  inv[4] = (h[0] * h[8] - h[2] * h[6]) / det;
  inv[5] = (h[2] * h[3] - h[0] * h[5]) / det;
  inv[6] = (h[3] * h[7] - h[4] * h[6]) / det;
  inv[7] = (h[1] * h[6] - h[0] * h[7]) / det;
  inv[8] = (h[0] * h[4] - h[1] * h[3]) / det;
  g->grid_ok = 1;
  for (int k = 0; k < 3; ++k) {
    double height = 1 / sqrt(inv[k] * inv[k] + inv[3 + k] * inv[3 + k] + inv[6 + k] * inv[6 + k]);
    double ratio = height / cutoff;
    g->grid_ok &= ratio >= 1;
    double dd = floor(ratio);
    g->dims[k] = (int)fmax(1.0, fmin((double)(0x7fffffff / 4), dd));
    double im = ceil(cutoff / height);
    if (im > 1000000) {
      seterr(err, cap, "Excessive periodic image range");
      return -1;
    }
    g->images[k] = im < 1 ? 1 : (int)im;
  }
  size_t capb = (size_t)(n < 1 ? 1 : n) * 8;
  if (capb > 64u * 1024 * 1024 / 16)
    capb = 64u * 1024 * 1024 / 16;
  while ((double)g->dims[0] * g->dims[1] * g->dims[2] > (double)capb) {
    int a = 0;
    for (int k = 1; k < 3; ++k)
      if (g->dims[k] > g->dims[a])
        a = k;
    g->dims[a] = (g->dims[a] + 1) / 2;
  }
  return 0;
}

/* Wrap exactly like the reference host loop: float32 wrapped positions and winding. */
static int wrap(const Geometry *g, int n, const float *xyz, float *w, int *wind, int *bin, char *err,
                int cap) {
  for (int i = 0; i < n; ++i) {
    double f[3];
    int b[3];
    for (int k = 0; k < 3; ++k) {
      double v = 0;
      for (int d = 0; d < 3; ++d) {
        float p = xyz[3 * i + d];
        if (!isfinite(p)) {
          seterr(err, cap, "Nonfinite coordinate");
          return -1;
        }
        v += p * g->inv[3 * d + k];
      }
      double fw = floor(v);
      if (fabs(fw) > 0x7fffffff / 4) {
        seterr(err, cap, "Coordinate winding exceeds int32 range");
        return -1;
      }
      wind[3 * i + k] = (int)fw;
      f[k] = v - fw;
      int bb = (int)(f[k] * g->dims[k]);
      b[k] = bb < g->dims[k] - 1 ? bb : g->dims[k] - 1;
    }
    for (int k = 0; k < 3; ++k)
      w[3 * i + k] = (float)(f[0] * g->h[k] + f[1] * g->h[3 + k] + f[2] * g->h[6 + k]);
    bin[i] = (b[0] * g->dims[1] + b[1]) * g->dims[2] + b[2];
  }
  return 0;
}

static int floor_div(int a, int b) {
  int q = a / b, r = a % b;
  return q - (r < 0);
}

static int edge_cmp(const void *pa, const void *pb) {
  const Edge *a = (const Edge *)pa, *b = (const Edge *)pb;
  int x[5] = {a->i, a->j, a->s[0], a->s[1], a->s[2]}, y[5] = {b->i, b->j, b->s[0], b->s[1], b->s[2]};
  for (int k = 0; k < 5; ++k)
    if (x[k] != y[k])
      return x[k] < y[k] ? -1 : 1;
  return 0;
}

typedef struct {
  Edge *e;
  int64_t n, cap;
} EdgeList;

static void push(EdgeList *l, Edge e) {
  if (l->n == l->cap) {
    l->cap = l->cap ? 2 * l->cap : 1024;
    l->e = (Edge *)realloc(l->e, (size_t)l->cap * sizeof(Edge));
  }
  l->e[l->n++] = e;
}

/* float32 displacement with the reference's operation order (no FMA contraction). */
static void consider(EdgeList *out, const float *w, const int *wind, const float *hf, float rc2, int i,
                     int j, int sx, int sy, int sz) {
  float d[3];
  for (int k = 0; k < 3; ++k)
    d[k] = w[3 * j + k] + (float)sx * hf[k] + (float)sy * hf[3 + k] + (float)sz * hf[6 + k] -
           w[3 * i + k];
  float r2 = d[0] * d[0] + d[1] * d[1] + d[2] * d[2];
  if (r2 <= rc2 && !(i == j && sx == 0 && sy == 0 && sz == 0)) {
    Edge e = {i, j, {sx + wind[3 * i] - wind[3 * j], sy + wind[3 * i + 1] - wind[3 * j + 1],
                     sz + wind[3 * i + 2] - wind[3 * j + 2]},
              {d[0], d[1], d[2]}};
    push(out, e);
  }
}

/* All directed edges (receiver i, sender j, caller-frame shift, float32 displacement),
 * sorted by (i, j, shift).  backend: 0 auto, 1 brute, 2 cell. */
static int enumerate(int n, const float *xyz, const float *cell, float cutoff, int backend, EdgeList *out,
                     char *err, int cap) {
  Geometry g;
  if (n < 0 || !isfinite(cutoff) || cutoff <= 0) {
    seterr(err, cap, "Invalid atom count or cutoff");
    return -1;
  }
  if (geometry(cell, cutoff, n, &g, err, cap))
    return -1;
  if (backend == 2 && !g.grid_ok) {
    seterr(err, cap, "CellList requires all reciprocal plane heights >= cutoff");
    return -1;
  }
  float *w = (float *)malloc(sizeof(float) * 3 * (n ? n : 1));
  int *wind = (int *)malloc(sizeof(int) * 3 * (n ? n : 1)), *bin = (int *)malloc(sizeof(int) * (n ? n : 1));
  if (wrap(&g, n, xyz, w, wind, bin, err, cap)) {
    free(w);
    free(wind);
    free(bin);
    return -1;
  }
  float hf[9], rc2 = cutoff * cutoff;
  for (int k = 0; k < 9; ++k)
    hf[k] = cell[k];
  out->n = 0;
  if (backend != 1 && g.grid_ok) {
    int nb = g.dims[0] * g.dims[1] * g.dims[2];
    int *start = (int *)calloc((size_t)nb + 1, sizeof(int)), *order = (int *)malloc(sizeof(int) * (n ? n : 1));
    for (int i = 0; i < n; ++i)
      start[bin[i] + 1]++;
    for (int b = 0; b < nb; ++b)
      start[b + 1] += start[b];
    int *fill = (int *)malloc(sizeof(int) * (size_t)(nb ? nb : 1));
    memcpy(fill, start, sizeof(int) * (size_t)nb);
    for (int i = 0; i < n; ++i)
      order[fill[bin[i]]++] = i;
    for (int i = 0; i < n; ++i) {
      int b = bin[i], bz = b % g.dims[2], by = (b / g.dims[2]) % g.dims[1], bx = b / (g.dims[1] * g.dims[2]);
      for (int x = -1; x <= 1; ++x)
        for (int y = -1; y <= 1; ++y)
          for (int z = -1; z <= 1; ++z) {
            int sx = floor_div(bx + x, g.dims[0]), sy = floor_div(by + y, g.dims[1]),
                sz = floor_div(bz + z, g.dims[2]);
            int c = ((bx + x - sx * g.dims[0]) * g.dims[1] + by + y - sy * g.dims[1]) * g.dims[2] + bz +
                    z - sz * g.dims[2];
            for (int q = start[c]; q < start[c + 1]; ++q)
              consider(out, w, wind, hf, rc2, i, order[q], sx, sy, sz);
          }
    }
    free(start);
    free(order);
    free(fill);
  } else {
    for (int i = 0; i < n; ++i)
      for (int x = -g.images[0]; x <= g.images[0]; ++x)
        for (int y = -g.images[1]; y <= g.images[1]; ++y)
          for (int z = -g.images[2]; z <= g.images[2]; ++z)
            for (int j = 0; j < n; ++j)
              consider(out, w, wind, hf, rc2, i, j, x, y, z);
  }
  qsort(out->e, (size_t)out->n, sizeof(Edge), edge_cmp);
  free(w);
  free(wind);
  free(bin);
  return 0;
}

/* Public: canonical edge list as 5 ints (i, j, sx, sy, sz) + 3 floats (d) per edge. */
int64_t oracle_edges(int n, const float *xyz, const float *cell, float cutoff, int backend, int64_t cap,
                     int *edges, float *disp, char *err, int errcap) {
  EdgeList l = {0};
  if (enumerate(n, xyz, cell, cutoff, backend, &l, err, errcap)) {
    free(l.e);
    return -1;
  }
  int64_t count = l.n;
  for (int64_t k = 0; k < count && k < cap; ++k) {
    int *o = edges + 5 * k;
    o[0] = l.e[k].i;
    o[1] = l.e[k].j;
    o[2] = l.e[k].s[0];
    o[3] = l.e[k].s[1];
    o[4] = l.e[k].s[2];
    if (disp)
      for (int q = 0; q < 3; ++q)
        disp[3 * k + q] = l.e[k].d[q];
  }
  free(l.e);
  return count;
}

/* ---------------- model math (double) ---------------- */
static double sigm(double x) { return 1 / (1 + exp(-x)); }

/* Linear: y[i][out_off + m*out_mul + co] (+)= sum_ci w[ci][co] x[i][in_off + m*in_mul + ci]. */
static void lin_fwd(const Lin *l, int n, const double *x, double *y, int add) {
#pragma omp parallel for schedule(static)
  for (int i = 0; i < n; ++i) {
    double *yi = y + (size_t)i * l->out;
    const double *xi = x + (size_t)i * l->in;
    if (!add)
      memset(yi, 0, sizeof(double) * (size_t)l->out);
    for (int q = 0; q < l->np; ++q) {
      Path p = l->p[q];
      const float *w = l->w + p.w_off;
      for (int m = 0; m < p.dim; ++m)
        for (int ci = 0; ci < p.in_mul; ++ci) {
          double v = xi[p.in_off + m * p.in_mul + ci];
          if (v == 0)
            continue;
          const float *wr = w + (size_t)ci * p.out_mul;
          double *yo = yi + p.out_off + m * p.out_mul;
          for (int co = 0; co < p.out_mul; ++co)
            yo[co] += v * wr[co];
        }
    }
  }
}
static void lin_bwd(const Lin *l, int n, const double *gy, double *gx, int add) {
#pragma omp parallel for schedule(static)
  for (int i = 0; i < n; ++i) {
    double *xi = gx + (size_t)i * l->in;
    const double *yi = gy + (size_t)i * l->out;
    if (!add)
      memset(xi, 0, sizeof(double) * (size_t)l->in);
    for (int q = 0; q < l->np; ++q) {
      Path p = l->p[q];
      const float *w = l->w + p.w_off;
      for (int m = 0; m < p.dim; ++m)
        for (int ci = 0; ci < p.in_mul; ++ci) {
          const float *wr = w + (size_t)ci * p.out_mul;
          const double *yo = yi + p.out_off + m * p.out_mul;
          double s = 0;
          for (int co = 0; co < p.out_mul; ++co)
            s += yo[co] * wr[co];
          xi[p.in_off + m * p.in_mul + ci] += s;
        }
    }
  }
}

/* Polynomial cutoff envelope and its r-derivative (mh1_math.cuh:34-40). */
static void envelope(double r, double rc, double p, double *v, double *dv) {
  if (r >= rc) {
    *v = *dv = 0;
    return;
  }
  double x = r / rc;
  double a = (p + 1) * (p + 2) * 0.5, b = p * (p + 2), c = p * (p + 1) * 0.5;
  *v = 1 - a * pow(x, p) + b * pow(x, p + 1) - c * pow(x, p + 2);
  *dv = (-a * p * pow(x, p - 1) + b * (p + 1) * pow(x, p) - c * (p + 2) * pow(x, p + 1)) / rc;
}

/* Component-normalised real harmonics of u = -d/r and dY/dd (mh1.cu:310-316). */
static void harmonics(const double d[3], double r, double Y[16], double G[16][3]) {
  double u[3] = {-d[0] / r, -d[1] / r, -d[2] / r};
  double x = u[0], y = u[1], z = u[2];
  double P[16], D[16][3];
  const double s3 = sqrt(3.0), s5 = sqrt(5.0), a9 = sqrt(5.0 / 6.0), a11 = sqrt(3.0 / 8.0);
  double xxzz = x * x + z * z, yy = y * y;
  double s4 = s3 * x * z, s8 = s3 / 2 * (z * z - x * x);
  double g4[3] = {s3 * z, 0, s3 * x}, g8[3] = {-s3 * x, 0, s3 * z};
  P[0] = 1;
  D[0][0] = D[0][1] = D[0][2] = 0;
  P[1] = x, P[2] = y, P[3] = z;
  for (int k = 0; k < 3; ++k)
    for (int q = 0; q < 3; ++q)
      D[1 + k][q] = k == q;
  P[4] = s4;
  memcpy(D[4], g4, sizeof g4);
  P[5] = s3 * x * y;
  D[5][0] = s3 * y, D[5][1] = s3 * x, D[5][2] = 0;
  P[6] = yy - 0.5 * xxzz;
  D[6][0] = -x, D[6][1] = 2 * y, D[6][2] = -z;
  P[7] = s3 * y * z;
  D[7][0] = 0, D[7][1] = s3 * z, D[7][2] = s3 * y;
  P[8] = s8;
  memcpy(D[8], g8, sizeof g8);
  P[9] = a9 * (s4 * z + s8 * x);
  for (int q = 0; q < 3; ++q)
    D[9][q] = a9 * (g4[q] * z + s4 * (q == 2) + g8[q] * x + s8 * (q == 0));
  P[10] = s5 * s4 * y;
  for (int q = 0; q < 3; ++q)
    D[10][q] = s5 * (g4[q] * y + s4 * (q == 1));
  double t = 4 * yy - xxzz, dt[3] = {-2 * x, 8 * y, -2 * z};
  P[11] = a11 * t * x;
  for (int q = 0; q < 3; ++q)
    D[11][q] = a11 * (dt[q] * x + t * (q == 0));
  double t2 = 2 * yy - 3 * xxzz, dt2[3] = {-6 * x, 4 * y, -6 * z};
  P[12] = 0.5 * y * t2;
  for (int q = 0; q < 3; ++q)
    D[12][q] = 0.5 * (t2 * (q == 1) + y * dt2[q]);
  P[13] = a11 * z * t;
  for (int q = 0; q < 3; ++q)
    D[13][q] = a11 * (t * (q == 2) + z * dt[q]);
  P[14] = s5 * s8 * y;
  for (int q = 0; q < 3; ++q)
    D[14][q] = s5 * (g8[q] * y + s8 * (q == 1));
  P[15] = a9 * (s8 * z - s4 * x);
  for (int q = 0; q < 3; ++q)
    D[15][q] = a9 * (g8[q] * z + s8 * (q == 2) - g4[q] * x - s4 * (q == 0));
  for (int k = 0; k < 16; ++k) {
    int l = k == 0 ? 0 : k < 4 ? 1 : k < 9 ? 2 : 3;
    double s = sqrt(2.0 * l + 1);
    Y[k] = s * P[k];
    /* dY/dd = sum_a dY/du_a du_a/dd, with du_a/dd_b = -(delta_ab - u_a u_b)/r */
    for (int b = 0; b < 3; ++b) {
      double g = 0;
      for (int a = 0; a < 3; ++a)
        g += D[k][a] * ((a == b) - u[a] * u[b]);
      G[k][b] = -s * g / r;
    }
  }
}

/* Radial hidden network with its r-tangent (mh1_math.cuh:121-173). */
static void radial_hidden(const Rad *w, int zs, int zr, const double in[NB], const double din[NB],
                          double h[HID], double dh[HID]) {
  double a[HID], da[HID];
  for (int t = 0; t < HID; ++t) {
    a[t] = (double)w->b0[t] + w->source[zs * 64 + t] + w->target[zr * 64 + t];
    da[t] = 0;
    for (int k = 0; k < NB; ++k) {
      a[t] += (double)w->radial[t * NB + k] * in[k];
      da[t] += (double)w->radial[t * NB + k] * din[k];
    }
  }
  for (int layer = 0; layer < w->depth; ++layer) {
    if (layer) {
      for (int t = 0; t < HID; ++t) {
        double s = w->bias[layer][t], ds = 0;
        for (int k = 0; k < HID; ++k) {
          s += (double)w->W[layer][t * 64 + k] * h[k];
          ds += (double)w->W[layer][t * 64 + k] * dh[k];
        }
        a[t] = s;
        da[t] = ds;
      }
    }
    double mean = 0, dmean = 0;
    for (int t = 0; t < HID; ++t)
      mean += a[t], dmean += da[t];
    mean /= HID, dmean /= HID;
    double var = 0, cov = 0;
    for (int t = 0; t < HID; ++t) {
      a[t] -= mean;
      da[t] -= dmean;
      var += a[t] * a[t];
      cov += a[t] * da[t];
    }
    double inv = 1 / sqrt(var / HID + 1e-5);
    double dinv = -inv * inv * inv * cov / HID;
    for (int t = 0; t < HID; ++t) {
      double g = w->gamma[layer][t];
      double u = a[t] * inv * g + w->beta[layer][t];
      double du = (da[t] * inv + a[t] * dinv) * g;
      double s = sigm(u);
      h[t] = u * s;
      dh[t] = du * s * (1 + u * (1 - s));
    }
  }
}

typedef struct {
  double r, cut, dcut, Y[16], G[16][3], in[NB], din[NB];
} EdgeGeom;

static void edge_geometry(const Model *m, const Edge *e, int zi, int zj, EdgeGeom *g) {
  double d[3] = {e->d[0], e->d[1], e->d[2]};
  double r = sqrt(d[0] * d[0] + d[1] * d[1] + d[2] * d[2]);
  if (r <= 0)
    r = 1e-10;
  g->r = r;
  double R = 0.5 * ((double)m->radii[zj] + m->radii[zi]);
  double ratio = r / R, dratio = 1 / R;
  double q = m->c[4], pp = m->c[5], a = m->c[3];
  /* transformed = 1 / (1 + a ratio^q / (1 + ratio^(q - p))) */
  double num = a * pow(ratio, q), dnum = a * q * pow(ratio, q - 1) * dratio;
  double den = 1 + pow(ratio, q - pp), dden = (q - pp) * pow(ratio, q - pp - 1) * dratio;
  double frac = num / den, dfrac = (dnum * den - num * dden) / (den * den);
  double t = 1 / (1 + frac), dt = -dfrac / ((1 + frac) * (1 + frac));
  envelope(r, m->c[0], m->c[2], &g->cut, &g->dcut);
  for (int k = 0; k < NB; ++k) {
    double wk = m->bessel[k];
    double v = m->c[1] * sin(wk * t) / t;
    double dv = m->c[1] * (wk * cos(wk * t) * t - sin(wk * t)) / (t * t) * dt;
    g->in[k] = v;
    g->din[k] = dv;
  }
  harmonics(d, r, g->Y, g->G);
}

/* ZBL pair repulsion, one directed edge: half energy, full receiver force, half virial. */
static void zbl(const Model *m, int zi, int zj, const Edge *e, double *energy, double f[3], double v[9]) {
  double d[3] = {e->d[0], e->d[1], e->d[2]};
  double r = sqrt(d[0] * d[0] + d[1] * d[1] + d[2] * d[2]);
  double rc = (double)m->zradii[zi] + m->zradii[zj];
  if (r <= 0 || r >= rc)
    return;
  double Zi = zi, Zj = zj;
  double a = m->c[9] * (double)0.529f / (pow(Zi, m->c[8]) + pow(Zj, m->c[8]));
  const double rates[4] = {3.2f, .9423f, .4028f, .2016f};
  double phi = 0, dphi = 0;
  for (int t = 0; t < 4; ++t) {
    double ex = exp(-rates[t] / a * r);
    phi += m->zc[t] * ex;
    dphi += -m->zc[t] * rates[t] / a * ex;
  }
  double env, denv;
  envelope(r, rc, m->c[10], &env, &denv);
  double pref = 0.5 * (double)14.3996f * Zi * Zj * m->c[6];
  double ev = pref * phi / r * env;
  double de = pref * ((dphi / r - phi / (r * r)) * env + phi / r * denv);
  *energy += ev;
  for (int k = 0; k < 3; ++k)
    f[k] += 2 * de * d[k] / r;
  for (int k = 0; k < 3; ++k)
    for (int l = 0; l < 3; ++l)
      v[3 * k + l] -= de * d[k] * d[l] / r;
}

static double *zeros(size_t n) { return (double *)calloc(n ? n : 1, sizeof(double)); }

static void debug_rms(const char *name, const double *x, size_t n) {
  if (!getenv("ORACLE_DEBUG"))
    return;
  double s = 0, mx = 0;
  for (size_t q = 0; q < n; ++q) {
    s += x[q] * x[q];
    mx = fmax(mx, fabs(x[q]));
  }
  fprintf(stderr, "oracle %-12s rms %.4g max %.4g\n", name, n ? sqrt(s / n) : 0.0, mx);
}

int oracle_threads(int n) {
#ifdef _OPENMP
  if (n > 0)
    omp_set_num_threads(n);
  return omp_get_max_threads();
#else
  (void)n;
  return 1;
#endif
}

/* Energy, per-atom energies, forces and virial for one structure (input order). */
int oracle_calculate(void *handle, int n, const float *xyz, const int *Z, const float *cell, int backend,
                     double *energy, double *atomic, double *force, double *virial, char *err, int errcap) {
  const Model *m = (const Model *)handle;
  if (!m || !energy || !virial || (n && (!xyz || !Z || !atomic || !force))) {
    seterr(err, errcap, "Null calculator or result pointer");
    return -1;
  }
  for (int i = 0; i < n; ++i)
    if (Z[i] < 1 || Z[i] > 118) {
      seterr(err, errcap, "Invalid atomic number");
      return -1;
    }
  EdgeList el = {0};
  if (enumerate(n, xyz, cell, 6.0f, backend, &el, err, errcap)) {
    free(el.e);
    return -1;
  }
  for (int i = 0; i < n; ++i)
    if (m->lookup[Z[i]] < 0) {
      free(el.e);
      seterr(err, errcap, "Model detected invalid device state (code 2)");
      return -1;
    }
  for (int64_t k = 0; k < el.n; ++k) {
    const Edge *e = &el.e[k];
    if (e->d[0] * e->d[0] + e->d[1] * e->d[1] + e->d[2] * e->d[2] <= 0) {
      free(el.e);
      seterr(err, errcap, "Model detected invalid device state (code 1)");
      return -1;
    }
  }
  int64_t ne = el.n;
  const Edge *E = el.e;
  int64_t *start = (int64_t *)calloc((size_t)n + 1, sizeof(int64_t));
  for (int64_t k = 0; k < ne; ++k)
    start[E[k].i + 1]++;
  for (int i = 0; i < n; ++i)
    start[i + 1] += start[i];
  const float *c = m->c;
  double *e = zeros((size_t)n), *F = zeros((size_t)3 * n), *V = zeros((size_t)9 * n);
  /* Embedding, shift and ZBL. */
  double *x0 = zeros((size_t)n * 512);
  for (int i = 0; i < n; ++i) {
    int s = m->lookup[Z[i]];
    for (int k = 0; k < 512; ++k)
      x0[(size_t)i * 512 + k] = m->emb[s * 512 + k];
    e[i] = c[7];
  }
  for (int64_t k = 0; k < ne; ++k)
    zbl(m, Z[E[k].i], Z[E[k].j], &E[k], &e[E[k].i], &F[3 * E[k].i], &V[9 * E[k].i]);
  EdgeGeom *G = (EdgeGeom *)malloc(sizeof(EdgeGeom) * (size_t)(ne ? ne : 1));
#pragma omp parallel for schedule(dynamic, 256)
  for (int64_t k = 0; k < ne; ++k)
    edge_geometry(m, &E[k], Z[E[k].i], Z[E[k].j], &G[k]);
  double *up[2], *res[2], *skip[2], *msg[2], *rho[2], *raw[2], *pre[2], *gate[2], *pin[2], *poly[2],
      *hidden[2];
  const double *input = x0;
  int in_dim = 512;
  for (int k = 0; k < 2; ++k) {
    const Layer *l = &m->L[k];
    int nc = l->out_comp, P = l->paths, hdim = k ? 512 : 2048;
    up[k] = zeros((size_t)n * l->in_comp * CH);
    res[k] = zeros((size_t)n * 9728);
    skip[k] = zeros((size_t)n * hdim);
    msg[k] = zeros((size_t)n * nc * CH);
    rho[k] = zeros((size_t)n);
    lin_fwd(&l->up, n, input, up[k], 0);
    lin_fwd(&l->res, n, up[k], res[k], 0);
    lin_fwd(&l->skip, n, input, skip[k], 0);
#pragma omp parallel
    {
      double *w = (double *)malloc(sizeof(double) * P * CH), h[HID], dh[HID], hd[HID], dhd[HID];
#pragma omp for schedule(dynamic, 4)
      for (int i = 0; i < n; ++i) {
        double *mi = msg[k] + (size_t)i * nc * CH;
        for (int64_t q = start[i]; q < start[i + 1]; ++q) {
          const Edge *ed = &E[q];
          const EdgeGeom *g = &G[q];
          int zs = m->lookup[Z[ed->j]], zr = m->lookup[Z[i]];
          radial_hidden(&l->radial, zs, zr, g->in, g->din, h, dh);
          for (int o = 0; o < P * CH; ++o) {
            double s = l->radial.ob[o];
            for (int a = 0; a < HID; ++a)
              s += (double)l->radial.ow[o * 64 + a] * h[a];
            w[o] = s * g->cut;
          }
          radial_hidden(&l->density, zs, zr, g->in, g->din, hd, dhd);
          double aa = l->density.ob[0];
          for (int a = 0; a < HID; ++a)
            aa += (double)l->density.ow[a] * hd[a];
          rho[k][i] += tanh(aa * aa) * g->cut;
          const double *uj = up[k] + (size_t)ed->j * l->in_comp * CH;
          for (int t = 0; t < l->nterms; ++t) {
            Term tt = l->tp[t];
            double f = (double)l->cg[t] * g->Y[tt.sh];
            const double *u = uj + tt.in * CH, *wp = w + tt.path * CH;
            double *o = mi + tt.out * CH;
            for (int ch = 0; ch < CH; ++ch)
              o[ch] += f * u[ch] * wp[ch];
          }
        }
      }
      free(w);
    }
    raw[k] = zeros((size_t)n * 9728);
    pre[k] = zeros((size_t)n * 9728);
    debug_rms("up", up[k], (size_t)n * l->in_comp * CH);
    debug_rms("res", res[k], (size_t)n * 9728);
    debug_rms("msg", msg[k], (size_t)n * nc * CH);
    debug_rms("rho", rho[k], (size_t)n);
    lin_fwd(&l->one, n, msg[k], raw[k], 0);
    for (int i = 0; i < n; ++i) {
      double den = l->alpha + l->beta * rho[k][i];
      for (int f = 0; f < 9728; ++f)
        pre[k][(size_t)i * 9728 + f] = raw[k][(size_t)i * 9728 + f] / den + res[k][(size_t)i * 9728 + f];
    }
    gate[k] = zeros((size_t)n * 8192);
    for (int i = 0; i < n; ++i) {
      const double *p = pre[k] + (size_t)i * 9728;
      double *g = gate[k] + (size_t)i * 8192;
      for (int ch = 0; ch < 512; ++ch) {
        double u = p[ch];
        g[ch] = c[11] * u * sigm(u);
        for (int L = 1; L <= 3; ++L) {
          double gl = sigm(p[L * 512 + ch]);
          for (int mm = L * L; mm < (L + 1) * (L + 1); ++mm)
            g[mm * 512 + ch] = p[2048 + (mm - 1) * 512 + ch] * c[12] * gl;
        }
      }
    }
    pin[k] = zeros((size_t)n * 8192);
    lin_fwd(&l->two, n, gate[k], pin[k], 0);
    poly[k] = zeros((size_t)n * l->pouts * 512);
#pragma omp parallel for schedule(static)
    for (int i = 0; i < n; ++i) {
      const double *x = pin[k] + (size_t)i * 8192;
      double *y = poly[k] + (size_t)i * l->pouts * 512;
      for (int t = 0; t < l->npoly; ++t) {
        Poly pq = l->poly[t];
        const float *w = l->pcoef + (size_t)t * 512;
        for (int ch = 0; ch < 512; ++ch) {
          double v = x[pq.a * 512 + ch];
          if (pq.deg >= 2)
            v *= x[pq.b * 512 + ch];
          if (pq.deg >= 3)
            v *= x[pq.c * 512 + ch];
          y[pq.out * 512 + ch] += (double)w[ch] * v;
        }
      }
    }
    hidden[k] = zeros((size_t)n * hdim);
    debug_rms("raw", raw[k], (size_t)n * 9728);
    debug_rms("pre", pre[k], (size_t)n * 9728);
    debug_rms("gate", gate[k], (size_t)n * 8192);
    debug_rms("pin", pin[k], (size_t)n * 8192);
    debug_rms("poly", poly[k], (size_t)n * l->pouts * 512);
    lin_fwd(&l->plin, n, poly[k], hidden[k], 0);
    for (size_t q = 0; q < (size_t)n * hdim; ++q)
      hidden[k][q] += skip[k][q];
    if (k == 0) {
      double *ne0 = zeros((size_t)n);
      lin_fwd(&m->read0, n, hidden[0], ne0, 0);
      for (int i = 0; i < n; ++i)
        e[i] += c[6] * ne0[i];
      free(ne0);
    }
    debug_rms("hidden", hidden[k], (size_t)n * hdim);
    input = hidden[k];
    in_dim = hdim;
  }
  (void)in_dim;
  double *rpre = zeros((size_t)n * 16), *rhid = zeros((size_t)n * 16), *ne1 = zeros((size_t)n);
  lin_fwd(&m->read1up, n, hidden[1], rpre, 0);
  for (size_t q = 0; q < (size_t)n * 16; ++q)
    rhid[q] = c[13] * rpre[q] * sigm(rpre[q]);
  lin_fwd(&m->read1down, n, rhid, ne1, 0);
  debug_rms("node_e1", ne1, (size_t)n);
  debug_rms("energy", e, (size_t)n);
  for (int i = 0; i < n; ++i)
    e[i] += c[6] * ne1[i];
  /* ---- analytical backward ---- */
  double *one = zeros((size_t)n), *rgrad = zeros((size_t)n * 16);
  for (int i = 0; i < n; ++i)
    one[i] = c[6];
  lin_bwd(&m->read1down, n, one, rgrad, 0);
  for (size_t q = 0; q < (size_t)n * 16; ++q) {
    double s = sigm(rpre[q]);
    rgrad[q] *= c[13] * s * (1 + rpre[q] * (1 - s));
  }
  double *hgrad = zeros((size_t)n * 512);
  lin_bwd(&m->read1up, n, rgrad, hgrad, 0);
  double *upgrad1 = NULL;
  for (int k = 1; k >= 0; --k) {
    const Layer *l = &m->L[k];
    int nc = l->out_comp, P = l->paths, hdim = k ? 512 : 2048;
    if (k == 0)
      lin_bwd(&m->read0, n, one, hgrad, 1);
    double *pgrad = zeros((size_t)n * l->pouts * 512);
    lin_bwd(&l->plin, n, hgrad, pgrad, 0);
    double *pingrad = zeros((size_t)n * 8192);
#pragma omp parallel for schedule(static)
    for (int i = 0; i < n; ++i) {
      const double *x = pin[k] + (size_t)i * 8192, *gy = pgrad + (size_t)i * l->pouts * 512;
      double *gx = pingrad + (size_t)i * 8192;
      for (int t = 0; t < l->npoly; ++t) {
        Poly pq = l->poly[t];
        const float *w = l->pcoef + (size_t)t * 512;
        for (int ch = 0; ch < 512; ++ch) {
          double g = (double)w[ch] * gy[pq.out * 512 + ch];
          double a = x[pq.a * 512 + ch], b = pq.deg >= 2 ? x[pq.b * 512 + ch] : 1,
                 d = pq.deg >= 3 ? x[pq.c * 512 + ch] : 1;
          gx[pq.a * 512 + ch] += g * b * d;
          if (pq.deg >= 2)
            gx[pq.b * 512 + ch] += g * a * d;
          if (pq.deg >= 3)
            gx[pq.c * 512 + ch] += g * a * b;
        }
      }
    }
    double *ggrad = zeros((size_t)n * 8192);
    lin_bwd(&l->two, n, pingrad, ggrad, 0);
    double *pregrad = zeros((size_t)n * 9728);
    for (int i = 0; i < n; ++i) {
      const double *p = pre[k] + (size_t)i * 9728, *gg = ggrad + (size_t)i * 8192;
      double *pg = pregrad + (size_t)i * 9728;
      for (int ch = 0; ch < 512; ++ch) {
        double u = p[ch], s = sigm(u);
        pg[ch] = gg[ch] * c[11] * s * (1 + u * (1 - s));
        for (int L = 1; L <= 3; ++L) {
          double gl = sigm(p[L * 512 + ch]), dg = 0;
          for (int mm = L * L; mm < (L + 1) * (L + 1); ++mm) {
            double src = p[2048 + (mm - 1) * 512 + ch];
            pg[2048 + (mm - 1) * 512 + ch] = gg[mm * 512 + ch] * c[12] * gl;
            dg += gg[mm * 512 + ch] * src * c[12] * gl * (1 - gl);
          }
          pg[L * 512 + ch] = dg;
        }
      }
    }
    double *rawgrad = zeros((size_t)n * 9728), *rhograd = zeros((size_t)n);
    for (int i = 0; i < n; ++i) {
      double den = l->alpha + l->beta * rho[k][i], s = 0;
      for (int f = 0; f < 9728; ++f) {
        double g = pregrad[(size_t)i * 9728 + f];
        rawgrad[(size_t)i * 9728 + f] = g / den;
        s -= g * raw[k][(size_t)i * 9728 + f] * l->beta / (den * den);
      }
      rhograd[i] = s;
    }
    double *msggrad = zeros((size_t)n * nc * CH);
    lin_bwd(&l->one, n, rawgrad, msggrad, 0);
    if (k == 1) {
      upgrad1 = zeros((size_t)n * l->in_comp * CH);
      lin_bwd(&l->res, n, pregrad, upgrad1, 0);
    }
    int nthreads = 1;
#ifdef _OPENMP
    nthreads = omp_get_max_threads();
#endif
    double **fpriv = (double **)calloc((size_t)nthreads, sizeof(double *));
    double **upriv = (double **)calloc((size_t)nthreads, sizeof(double *));
#pragma omp parallel
    {
      int tid = 0;
#ifdef _OPENMP
      tid = omp_get_thread_num();
#endif
      fpriv[tid] = zeros((size_t)3 * n);
      if (k == 1)
        upriv[tid] = zeros((size_t)n * l->in_comp * CH);
      double *w = (double *)malloc(sizeof(double) * P * CH), *dw = (double *)malloc(sizeof(double) * P * CH);
      double h[HID], dh[HID], hd[HID], dhd[HID];
#pragma omp for schedule(dynamic, 4)
      for (int i = 0; i < n; ++i) {
        const double *gi = msggrad + (size_t)i * nc * CH;
        for (int64_t q = start[i]; q < start[i + 1]; ++q) {
          const Edge *ed = &E[q];
          const EdgeGeom *g = &G[q];
          int zs = m->lookup[Z[ed->j]], zr = m->lookup[Z[i]];
          radial_hidden(&l->radial, zs, zr, g->in, g->din, h, dh);
          for (int o = 0; o < P * CH; ++o) {
            double s = l->radial.ob[o], ds = 0;
            for (int a = 0; a < HID; ++a) {
              s += (double)l->radial.ow[o * 64 + a] * h[a];
              ds += (double)l->radial.ow[o * 64 + a] * dh[a];
            }
            w[o] = s * g->cut;
            dw[o] = ds * g->cut + s * g->dcut;
          }
          radial_hidden(&l->density, zs, zr, g->in, g->din, hd, dhd);
          double aa = l->density.ob[0], daa = 0;
          for (int a = 0; a < HID; ++a) {
            aa += (double)l->density.ow[a] * hd[a];
            daa += (double)l->density.ow[a] * dhd[a];
          }
          double th = tanh(aa * aa);
          double dden = 2 * aa * daa * (1 - th * th) * g->cut + th * g->dcut;
          const double *uj = up[k] + (size_t)ed->j * l->in_comp * CH;
          double dr = rhograd[i] * dden, gv[3] = {0, 0, 0};
          for (int t = 0; t < l->nterms; ++t) {
            Term tt = l->tp[t];
            const double *u = uj + tt.in * CH, *wp = w + tt.path * CH, *dwp = dw + tt.path * CH,
                         *gg = gi + tt.out * CH;
            double cg = l->cg[t], Yv = g->Y[tt.sh];
            double suw = 0, sudw = 0;
            for (int ch = 0; ch < CH; ++ch) {
              double a = gg[ch] * cg;
              suw += a * u[ch] * wp[ch];
              sudw += a * u[ch] * dwp[ch];
              if (k == 1)
                upriv[tid][((size_t)ed->j * l->in_comp + tt.in) * CH + ch] += a * Yv * wp[ch];
            }
            dr += Yv * sudw;
            for (int b = 0; b < 3; ++b)
              gv[b] += suw * g->G[tt.sh][b];
          }
          double f[3];
          for (int b = 0; b < 3; ++b) {
            f[b] = gv[b] + dr * ed->d[b] / g->r;
            F[3 * i + b] += f[b];
            fpriv[tid][3 * ed->j + b] -= f[b];
          }
          for (int a = 0; a < 3; ++a)
            for (int b = 0; b < 3; ++b)
              V[9 * i + 3 * a + b] -= (double)ed->d[a] * f[b];
        }
      }
      free(w);
      free(dw);
    }
    for (int t = 0; t < nthreads; ++t) {
      if (fpriv[t]) {
        for (size_t q = 0; q < (size_t)3 * n; ++q)
          F[q] += fpriv[t][q];
        free(fpriv[t]);
      }
      if (upriv[t]) {
        for (size_t q = 0; q < (size_t)n * l->in_comp * CH; ++q)
          upgrad1[q] += upriv[t][q];
        free(upriv[t]);
      }
    }
    free(fpriv);
    free(upriv);
    if (k == 1) {
      double *prev = zeros((size_t)n * 2048);
      lin_bwd(&l->skip, n, hgrad, prev, 0);
      lin_bwd(&l->up, n, upgrad1, prev, 1);
      free(hgrad);
      hgrad = prev;
    }
    free(pgrad);
    free(pingrad);
    free(ggrad);
    free(pregrad);
    free(rawgrad);
    free(rhograd);
    free(msggrad);
    (void)hdim;
  }
  double total = 0;
  for (int i = 0; i < n; ++i) {
    double base = m->e0[Z[i]];
    atomic[i] = e[i] + base;
    total += e[i] + base;
    for (int b = 0; b < 3; ++b)
      force[3 * i + b] = F[3 * i + b];
  }
  *energy = total;
  for (int q = 0; q < 9; ++q) {
    double s = 0;
    for (int i = 0; i < n; ++i)
      s += V[9 * i + q];
    virial[q] = s;
  }
  free(upgrad1);
  free(hgrad);
  free(one);
  free(rgrad);
  free(rpre);
  free(rhid);
  free(ne1);
  for (int k = 0; k < 2; ++k) {
    free(up[k]), free(res[k]), free(skip[k]), free(msg[k]), free(rho[k]), free(raw[k]);
    free(pre[k]), free(gate[k]), free(pin[k]), free(poly[k]), free(hidden[k]);
  }
  free(G);
  free(x0);
  free(e);
  free(F);
  free(V);
  free(start);
  free(el.e);
  return 0;
}
