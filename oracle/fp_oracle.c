/*
 * TEST INFRASTRUCTURE ONLY -- CPU restatement of the reference hot path.
 * See fp_oracle.h for scope and who may call it. Every function cites the
 * reference file:line whose arithmetic it restates; citations are paths inside
 * the nvidia-isaac/foundation-pose-inference-library project.
 */
#include "fp_oracle.h"

#include <float.h>
#include <limits.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>

typedef struct { float x, y, z; } f3;
typedef struct { float x, y, z, w; } f4;

static f3 mk3(float x, float y, float z) { f3 r = {x, y, z}; return r; }
static int imin(int a, int b) { return a < b ? a : b; }
static int imax(int a, int b) { return a > b ? a : b; }
static float clampf(float v, float lo, float hi) { return fminf(fmaxf(v, lo), hi); }
/* __saturatef: clamp to [0,1], NaN -> 0. */
static float saturatef(float v) { return v != v ? 0.0f : clampf(v, 0.0f, 1.0f); }

/* config.hpp:20-67 defaults. */
void fpo_default_config(fpo_config* c) {
  c->depth_min = 0.001f;
  c->depth_max = 100.0f;
  c->erosion_radius = 2;
  c->bilateral_radius = 2;
  c->depth_diff_threshold = 0.001f;
  c->erosion_ratio_threshold = 0.8f;
  c->bilateral_sigma_d = 2.0f;
  c->bilateral_sigma_r = 100000.0f;
  c->crop_ratio = 1.2f;
  c->input_width = 160;
  c->input_height = 160;
  c->rotation_normalizer_rad = 0.3490658503988659f;
  c->znear = 0.001f;
  c->zfar = 100.0f;
  c->ambient_weight = 0.8f;
  c->diffuse_weight = 0.5f;
}

/* cuda_pipeline.cu:30-32 validDepth. */
static int valid_depth(float z, const fpo_config* c) {
  return isfinite(z) && z >= c->depth_min && z < c->depth_max;
}

/* cuda_pipeline.cu:87-120 erodeDepthKernel: in-bounds neighbours only. */
void fpo_erode(const float* in, float* out, int w, int h, const fpo_config* c) {
  const int radius = imax(c->erosion_radius, 0);
  for (int y = 0; y < h; ++y) {
    for (int x = 0; x < w; ++x) {
      const int idx = y * w + x;
      const float center = in[idx];
      if (!valid_depth(center, c)) {
        out[idx] = 0.0f;
        continue;
      }
      int bad = 0, total = 0;
      for (int yy = imax(0, y - radius); yy <= imin(h - 1, y + radius); ++yy) {
        for (int xx = imax(0, x - radius); xx <= imin(w - 1, x + radius); ++xx) {
          const float z = in[yy * w + xx];
          ++total;
          if (!valid_depth(z, c) || fabsf(z - center) > c->depth_diff_threshold) ++bad;
        }
      }
      out[idx] = (total > 0 && (float)bad / (float)total > c->erosion_ratio_threshold) ? 0.0f
                                                                                      : center;
    }
  }
}

/* cuda_pipeline.cu:122-171 bilateralDepthKernel. */
void fpo_bilateral(const float* in, float* out, int w, int h, const fpo_config* c) {
  const int radius = imax(c->bilateral_radius, 0);
  const float sigma_d2 = 2.0f * c->bilateral_sigma_d * c->bilateral_sigma_d;
  const float sigma_r2 = 2.0f * c->bilateral_sigma_r * c->bilateral_sigma_r;
  for (int y = 0; y < h; ++y) {
    for (int x = 0; x < w; ++x) {
      float mean = 0.0f;
      int valid = 0;
      for (int yy = imax(0, y - radius); yy <= imin(h - 1, y + radius); ++yy)
        for (int xx = imax(0, x - radius); xx <= imin(w - 1, x + radius); ++xx) {
          const float z = in[yy * w + xx];
          if (valid_depth(z, c)) {
            mean += z;
            ++valid;
          }
        }
      const int idx = y * w + x;
      if (valid == 0) {
        out[idx] = 0.0f;
        continue;
      }
      mean /= (float)valid;
      float weighted = 0.0f, weight_sum = 0.0f;
      for (int yy = imax(0, y - radius); yy <= imin(h - 1, y + radius); ++yy)
        for (int xx = imax(0, x - radius); xx <= imin(w - 1, x + radius); ++xx) {
          const float z = in[yy * w + xx];
          if (!valid_depth(z, c)) continue;
          const float dx = (float)(xx - x);
          const float dy = (float)(yy - y);
          const float range = z - mean;
          const float wgt = expf(-(dx * dx + dy * dy) / sigma_d2) * expf(-(range * range) / sigma_r2);
          weighted += wgt * z;
          weight_sum += wgt;
        }
      out[idx] = weight_sum > 0.0f ? weighted / weight_sum : 0.0f;
    }
  }
}

/* cuda_pipeline.cu:173-192 depthToXyzKernel. k4 = fx, fy, cx, cy. */
void fpo_depth_to_xyz(const float* depth, float* xyz, int w, int h, const float* k4,
                      const fpo_config* c) {
  for (int y = 0; y < h; ++y)
    for (int x = 0; x < w; ++x) {
      const int idx = y * w + x;
      const float z = depth[idx];
      if (!valid_depth(z, c)) {
        xyz[3 * idx] = xyz[3 * idx + 1] = xyz[3 * idx + 2] = 0.0f;
        continue;
      }
      xyz[3 * idx + 0] = ((float)x - k4[2]) * z / k4[0];
      xyz[3 * idx + 1] = ((float)y - k4[3]) * z / k4[1];
      xyz[3 * idx + 2] = z;
    }
}

/* pipeline_utils.cpp:250-263 preprocessDepth with erodeDepth :31-69 (out-of-bounds
 * neighbours count as bad; fixed denominator) and bilateralFilter :71-139. */
void fpo_preprocess_cpu(const float* depth, float* out, int w, int h, const fpo_config* c) {
  const size_t n = (size_t)w * h;
  float* clamped = (float*)malloc(n * sizeof(float));
  float* eroded = (float*)calloc(n, sizeof(float));
  for (size_t i = 0; i < n; ++i) {
    const float z = depth[i];
    clamped[i] = (z < c->depth_min || z >= c->depth_max || !isfinite(z)) ? 0.0f : z;
  }
  const int radius = imax(c->erosion_radius, 0);
  const int kernel = 2 * radius + 1;
  const float denom = (float)(kernel * kernel);
  for (int y = 0; y < h; ++y)
    for (int x = 0; x < w; ++x) {
      const float center = clamped[(size_t)y * w + x];
      const int center_invalid = center < c->depth_min || center >= c->depth_max;
      int bad = 0;
      for (int dy = -radius; dy <= radius; ++dy)
        for (int dx = -radius; dx <= radius; ++dx) {
          const int xx = x + dx, yy = y + dy;
          float nb = 0.0f;
          if (xx >= 0 && yy >= 0 && xx < w && yy < h) nb = clamped[(size_t)yy * w + xx];
          if (nb < c->depth_min || nb >= c->depth_max || fabsf(nb - center) > c->depth_diff_threshold)
            ++bad;
        }
      if (!center_invalid && (float)bad / denom <= c->erosion_ratio_threshold)
        eroded[(size_t)y * w + x] = center;
    }
  /* bilateralFilter: spatial weights precomputed with expf in row-major tap order. */
  const int br = imax(c->bilateral_radius, 0);
  const int taps = (2 * br + 1) * (2 * br + 1);
  float* spatial = (float*)malloc((size_t)taps * sizeof(float));
  int k = 0;
  for (int dy = -br; dy <= br; ++dy)
    for (int dx = -br; dx <= br; ++dx)
      spatial[k++] = expf(-(float)(dx * dx + dy * dy) /
                          (2.0f * c->bilateral_sigma_d * c->bilateral_sigma_d));
  memset(out, 0, n * sizeof(float));
  for (int y = 0; y < h; ++y)
    for (int x = 0; x < w; ++x) {
      float mean = 0.0f;
      int vc = 0;
      for (int dy = -br; dy <= br; ++dy)
        for (int dx = -br; dx <= br; ++dx) {
          const int xx = x + dx, yy = y + dy;
          if (xx < 0 || yy < 0 || xx >= w || yy >= h) continue;
          const float z = eroded[(size_t)yy * w + xx];
          if (z >= c->depth_min && z < c->depth_max) {
            mean += z;
            ++vc;
          }
        }
      if (vc == 0) continue;
      mean /= (float)vc;
      float weighted = 0.0f, wsum = 0.0f;
      k = 0;
      for (int dy = -br; dy <= br; ++dy)
        for (int dx = -br; dx <= br; ++dx, ++k) {
          const int xx = x + dx, yy = y + dy;
          if (xx < 0 || yy < 0 || xx >= w || yy >= h) continue;
          const float z = eroded[(size_t)yy * w + xx];
          if (z < c->depth_min || z >= c->depth_max) continue;
          const float range = z - mean;
          const float wr = expf(-(range * range) / (2.0f * c->bilateral_sigma_r * c->bilateral_sigma_r));
          const float wt = spatial[k] * wr;
          weighted += wt * z;
          wsum += wt;
        }
      if (wsum > 0.0f) out[(size_t)y * w + x] = weighted / wsum;
    }
  free(spatial);
  free(eroded);
  free(clamped);
}

#define FPO_HIST_BINS 65536

/* cuda_pipeline.cu:194-299 computeBlockStats + depthHistogram + finalizeTranslation:
 * mask bbox, count of valid masked depth, 65,536-bin histogram median. */
void fpo_initial_translation(const float* depth, const uint8_t* mask, int w, int h,
                             const float* k4, const fpo_config* c, float* t3) {
  int min_x = INT_MAX, max_x = -1, min_y = INT_MAX, max_y = -1, count = 0;
  int* hist = (int*)calloc(FPO_HIST_BINS, sizeof(int));
  for (int y = 0; y < h; ++y)
    for (int x = 0; x < w; ++x) {
      const int idx = y * w + x;
      if (mask[idx] == 0) continue;
      min_x = imin(min_x, x);
      max_x = imax(max_x, x);
      min_y = imin(min_y, y);
      max_y = imax(max_y, y);
      const float z = depth[idx];
      if (!valid_depth(z, c)) continue;
      ++count;
      const float normalized = (z - c->depth_min) / (c->depth_max - c->depth_min);
      const int bin = imin(imax((int)(normalized * FPO_HIST_BINS), 0), FPO_HIST_BINS - 1);
      hist[bin] += 1;
    }
  if (max_x < min_x || count <= 0) {
    t3[0] = t3[1] = t3[2] = 0.0f;
    free(hist);
    return;
  }
  int cumulative = 0, median_bin = 0;
  const int median_rank = count / 2;
  for (int bin = 0; bin < FPO_HIST_BINS; ++bin) {
    cumulative += hist[bin];
    if (cumulative > median_rank) {
      median_bin = bin;
      break;
    }
  }
  free(hist);
  const float z_range = c->depth_max - c->depth_min;
  const float z = c->depth_min + ((float)median_bin + 0.5f) * z_range / (float)FPO_HIST_BINS;
  const float u = 0.5f * ((float)min_x + (float)max_x);
  const float v = 0.5f * ((float)min_y + (float)max_y);
  t3[0] = (u - k4[2]) * z / k4[0];
  t3[1] = (v - k4[3]) * z / k4[1];
  t3[2] = z;
}

static int cmp_float(const void* a, const void* b) {
  const float fa = *(const float*)a, fb = *(const float*)b;
  return (fa > fb) - (fa < fb);
}

/* pipeline_utils.cpp:288-332 guessTranslation: exact median via nth_element. */
void fpo_guess_translation_cpu(const float* depth, const uint8_t* mask, int w, int h,
                               const float* k4, const fpo_config* c, float* t3) {
  int min_x = w, max_x = -1, min_y = h, max_y = -1;
  float* vals = (float*)malloc((size_t)w * h * sizeof(float));
  size_t nv = 0;
  for (int y = 0; y < h; ++y)
    for (int x = 0; x < w; ++x) {
      const size_t idx = (size_t)y * w + x;
      if (mask[idx] == 0) continue;
      min_x = imin(min_x, x);
      max_x = imax(max_x, x);
      min_y = imin(min_y, y);
      max_y = imax(max_y, y);
      const float z = depth[idx];
      if (z >= c->depth_min && z < c->depth_max) vals[nv++] = z;
    }
  if (max_x < min_x || nv == 0) {
    t3[0] = t3[1] = t3[2] = 0.0f;
    free(vals);
    return;
  }
  qsort(vals, nv, sizeof(float), cmp_float);
  const float z = vals[nv / 2];
  free(vals);
  const float u = ((float)min_x + (float)max_x) * 0.5f;
  const float v = ((float)min_y + (float)max_y) * 0.5f;
  t3[0] = (u - k4[2]) * z / k4[0];
  t3[1] = (v - k4[3]) * z / k4[1];
  t3[2] = z;
}

/* ---- rotation grid: pipeline_utils.cpp:141-246 with math_utils.hpp helpers ---- */

static float dot3(f3 a, f3 b) { return a.x * b.x + a.y * b.y + a.z * b.z; }
static f3 cross3(f3 a, f3 b) {
  return mk3(a.y * b.z - a.z * b.y, a.z * b.x - a.x * b.z, a.x * b.y - a.y * b.x);
}
static float norm3(f3 a) { return sqrtf(fmaxf(dot3(a, a), 0.0f)); }
/* math_utils.hpp:497-503 normalize (zero vector for tiny norms). */
static f3 normalize_host(f3 a) {
  const float n = norm3(a);
  if (n < 1e-12f) return mk3(0.0f, 0.0f, 0.0f);
  return mk3(a.x / n, a.y / n, a.z / n);
}
static void mat3_mul(const float* a, const float* b, float* out) {
  for (int r = 0; r < 3; ++r)
    for (int c = 0; c < 3; ++c) {
      float v = 0.0f;
      for (int k = 0; k < 3; ++k) v += a[r * 3 + k] * b[k * 3 + c];
      out[r * 3 + c] = v;
    }
}
static void mat3_transpose(const float* m, float* out) {
  for (int r = 0; r < 3; ++r)
    for (int c = 0; c < 3; ++c) out[r * 3 + c] = m[c * 3 + r];
}

typedef struct { int a, b, c; } tri3;

/* pipeline_utils.cpp:141-154 midpoint with an edge cache keyed by (min, max). */
static int midpoint(int a, int b, f3* verts, int* nverts, int* keys, int* vals, int* nkeys) {
  const int lo = imin(a, b), hi = imax(a, b);
  for (int i = 0; i < *nkeys; ++i)
    if (keys[2 * i] == lo && keys[2 * i + 1] == hi) return vals[i];
  f3 s = mk3((verts[a].x + verts[b].x) * 0.5f, (verts[a].y + verts[b].y) * 0.5f,
             (verts[a].z + verts[b].z) * 0.5f);
  const int idx = (*nverts)++;
  verts[idx] = normalize_host(s);
  keys[2 * *nkeys] = lo;
  keys[2 * *nkeys + 1] = hi;
  vals[(*nkeys)++] = idx;
  return idx;
}

/* pipeline_utils.cpp:156-190 sampleIcosphere(min_vertices); returns vertex count. */
static int sample_icosphere(int min_vertices, f3** out) {
  const float t = (1.0f + sqrtf(5.0f)) * 0.5f;
  const f3 base[12] = {{-1, t, 0}, {1, t, 0}, {-1, -t, 0}, {1, -t, 0}, {0, -1, t}, {0, 1, t},
                       {0, -1, -t}, {0, 1, -t}, {t, 0, -1}, {t, 0, 1}, {-t, 0, -1}, {-t, 0, 1}};
  static const int base_faces[20][3] = {{0, 11, 5}, {0, 5, 1},  {0, 1, 7},   {0, 7, 10}, {0, 10, 11},
                                        {1, 5, 9},  {5, 11, 4}, {11, 10, 2}, {10, 7, 6}, {7, 1, 8},
                                        {3, 9, 4},  {3, 4, 2},  {3, 2, 6},   {3, 6, 8},  {3, 8, 9},
                                        {4, 9, 5},  {2, 4, 11}, {6, 2, 10},  {8, 6, 7},  {9, 8, 1}};
  int cap = 12, nv = 12, nf = 20;
  f3* verts = (f3*)malloc(sizeof(f3) * cap);
  for (int i = 0; i < 12; ++i) verts[i] = normalize_host(base[i]);
  tri3* faces = (tri3*)malloc(sizeof(tri3) * nf);
  for (int i = 0; i < nf; ++i) {
    faces[i].a = base_faces[i][0];
    faces[i].b = base_faces[i][1];
    faces[i].c = base_faces[i][2];
  }
  while (nv < min_vertices) {
    cap = nv + 3 * nf;
    verts = (f3*)realloc(verts, sizeof(f3) * cap);
    int* keys = (int*)malloc(sizeof(int) * 2 * 3 * nf);
    int* vals = (int*)malloc(sizeof(int) * 3 * nf);
    int nkeys = 0;
    tri3* next = (tri3*)malloc(sizeof(tri3) * 4 * nf);
    for (int i = 0; i < nf; ++i) {
      const tri3 f = faces[i];
      const int ab = midpoint(f.a, f.b, verts, &nv, keys, vals, &nkeys);
      const int bc = midpoint(f.b, f.c, verts, &nv, keys, vals, &nkeys);
      const int ca = midpoint(f.c, f.a, verts, &nv, keys, vals, &nkeys);
      next[4 * i + 0] = (tri3){f.a, ab, ca};
      next[4 * i + 1] = (tri3){f.b, bc, ab};
      next[4 * i + 2] = (tri3){f.c, ca, bc};
      next[4 * i + 3] = (tri3){ab, bc, ca};
    }
    free(keys);
    free(vals);
    free(faces);
    faces = next;
    nf *= 4;
  }
  free(faces);
  *out = verts;
  return nv;
}

/* pipeline_utils.cpp:192-213 cameraInObjectFromView, then rotation part and
 * translation; math_utils.hpp:597-602 inverseRigid; :604-613 rotationZ;
 * :640-645 geodesicDistance. */
int fpo_rotation_grid(float* out9, int max_count) {
  const int min_n_views = 40;
  const float inplane_step_deg = 60.0f;
  const float cluster_threshold_deg = 30.0f;
  const float kPi = 3.14159265358979323846f;
  f3* views = NULL;
  const int nviews = sample_icosphere(min_n_views, &views);
  int n_inplane = (int)roundf(360.0f / inplane_step_deg);
  if (n_inplane < 1) n_inplane = 1;
  const float step = inplane_step_deg * kPi / 180.0f;
  const int total = nviews * n_inplane;
  float* rots = (float*)malloc(sizeof(float) * 9 * total);
  int nr = 0;
  for (int vi = 0; vi < nviews; ++vi) {
    const f3 cam_pos = views[vi];
    const f3 z_axis = normalize_host(mk3(cam_pos.x * -1.0f, cam_pos.y * -1.0f, cam_pos.z * -1.0f));
    f3 x_axis = cross3(mk3(0.0f, 0.0f, 1.0f), z_axis);
    if (norm3(x_axis) < 0.001f) x_axis = mk3(1.0f, 0.0f, 0.0f);
    x_axis = normalize_host(x_axis);
    const f3 y_axis = normalize_host(cross3(z_axis, x_axis));
    /* base_r columns are the camera axes expressed in the object frame. */
    const float base_r[9] = {x_axis.x, y_axis.x, z_axis.x, x_axis.y, y_axis.y,
                             z_axis.y, x_axis.z, y_axis.z, z_axis.z};
    for (int j = 0; j < n_inplane; ++j) {
      const float theta = (float)j * step;
      const float cz = cosf(theta), sz = sinf(theta);
      const float rz[9] = {cz, -sz, 0.0f, sz, cz, 0.0f, 0.0f, 0.0f, 1.0f};
      float cam_r[9];
      mat3_mul(base_r, rz, cam_r);
      /* obj_in_cam rotation = transpose(cam_r); the translation does not
       * affect the rotation part. */
      mat3_transpose(cam_r, rots + 9 * nr);
      ++nr;
    }
  }
  free(views);
  const float threshold = cluster_threshold_deg * kPi / 180.0f;
  int nc = 0;
  for (int i = 0; i < nr; ++i) {
    const float* cand = rots + 9 * i;
    int is_new = 1;
    for (int j = 0; j < nc; ++j) {
      const float* ex = rots + 9 * j; /* clustered entries are compacted to the front */
      float bt[9], rel[9];
      mat3_transpose(ex, bt);
      mat3_mul(cand, bt, rel);
      const float trace = rel[0] + rel[4] + rel[8];
      const float cos_theta = clampf((trace - 1.0f) * 0.5f, -1.0f, 1.0f);
      if (acosf(cos_theta) < threshold) {
        is_new = 0;
        break;
      }
    }
    if (is_new) {
      if (nc != i) memmove(rots + 9 * nc, cand, 9 * sizeof(float));
      ++nc;
    }
  }
  for (int i = 0; i < nc && i < max_count; ++i) memcpy(out9 + 9 * i, rots + 9 * i, 9 * sizeof(float));
  free(rots);
  return nc;
}

/* cuda_pipeline.cu:301-327 seedPosesKernel. */
void fpo_seed_poses(const float* r9, const float* t3, int n, float* p) {
  for (int i = 0; i < n; ++i) {
    const float* r = r9 + 9 * i;
    float* q = p + 16 * i;
    q[0] = r[0]; q[1] = r[1]; q[2] = r[2]; q[3] = t3[0];
    q[4] = r[3]; q[5] = r[4]; q[6] = r[5]; q[7] = t3[1];
    q[8] = r[6]; q[9] = r[7]; q[10] = r[8]; q[11] = t3[2];
    q[12] = 0.0f; q[13] = 0.0f; q[14] = 0.0f; q[15] = 1.0f;
  }
}

/* cuda_pipeline.cu:329-368 cropBoxesKernel. */
void fpo_crop_boxes(const float* poses, int n, const float* k4, float diameter,
                    const fpo_config* c, float* boxes) {
  for (int i = 0; i < n; ++i) {
    const float* pose = poses + 16 * i;
    const f3 center = mk3(pose[3], pose[7], pose[11]);
    const float radius = diameter * c->crop_ratio * 0.5f;
    const f3 off[5] = {{0, 0, 0}, {radius, 0, 0}, {-radius, 0, 0}, {0, radius, 0}, {0, -radius, 0}};
    float cu = 0.0f, cv = 0.0f, rpx = 1.0f;
    for (int j = 0; j < 5; ++j) {
      const f3 p = mk3(center.x + off[j].x, center.y + off[j].y, center.z + off[j].z);
      const float inv_z = fabsf(p.z) > 1e-12f ? 1.0f / p.z : 0.0f;
      const float u = k4[0] * p.x * inv_z + k4[2];
      const float v = k4[1] * p.y * inv_z + k4[3];
      if (j == 0) {
        cu = u;
        cv = v;
      } else {
        rpx = fmaxf(rpx, fabsf(u - cu));
        rpx = fmaxf(rpx, fabsf(v - cv));
      }
    }
    boxes[4 * i + 0] = roundf(cu - rpx);
    boxes[4 * i + 1] = roundf(cv - rpx);
    boxes[4 * i + 2] = roundf(cu + rpx);
    boxes[4 * i + 3] = roundf(cv + rpx);
  }
}

/* raster_kernels.cuh:324-330 normalize3 (fallback +z). */
static f3 normalize3(f3 v) {
  const float n = sqrtf(fmaxf(v.x * v.x + v.y * v.y + v.z * v.z, 0.0f));
  if (n < 1e-12f) return mk3(0.0f, 0.0f, 1.0f);
  return mk3(v.x / n, v.y / n, v.z / n);
}

/* builtin_raster_renderer.cu:28-33 packDepthKey. */
static uint64_t pack_depth_key(float zw, int tri_plus_one) {
  const float d01 = fminf(fmaxf(zw * 0.5f + 0.5f, 0.0f), 1.0f);
  uint32_t bits;
  memcpy(&bits, &d01, 4);
  return ((uint64_t)bits << 32) | (uint32_t)tri_plus_one;
}

/* raster_kernels.cuh:336-380 buildRenderVerticesKernel for one hypothesis. */
static void build_vertices(const float* verts, const float* normals, int nv, const float* pose,
                           const float* box, const float* k4, const fpo_config* c, f4* clip,
                           f3* cam_pos, f3* cam_nrm) {
  for (int i = 0; i < nv; ++i) {
    const f3 p = mk3(verts[3 * i], verts[3 * i + 1], verts[3 * i + 2]);
    const f3 n = mk3(normals[3 * i], normals[3 * i + 1], normals[3 * i + 2]);
    const f3 cam = mk3(pose[0] * p.x + pose[1] * p.y + pose[2] * p.z + pose[3],
                       pose[4] * p.x + pose[5] * p.y + pose[6] * p.z + pose[7],
                       pose[8] * p.x + pose[9] * p.y + pose[10] * p.z + pose[11]);
    cam_nrm[i] = normalize3(mk3(pose[0] * n.x + pose[1] * n.y + pose[2] * n.z,
                                pose[4] * n.x + pose[5] * n.y + pose[6] * n.z,
                                pose[8] * n.x + pose[9] * n.y + pose[10] * n.z));
    cam_pos[i] = cam;
    const float z = fmaxf(cam.z, c->znear);
    const float u = k4[0] * cam.x / z + k4[2];
    const float v = k4[1] * cam.y / z + k4[3];
    const float crop_w = fmaxf(box[2] - box[0], 1.0f);
    const float crop_h = fmaxf(box[3] - box[1], 1.0f);
    const float ndc_x = 2.0f * (u - box[0]) / crop_w - 1.0f;
    const float ndc_y = 1.0f - 2.0f * (v - box[1]) / crop_h;
    const float depth = c->zfar - c->znear;
    const float clip_z = ((c->zfar + c->znear) / depth) * z - (2.0f * c->zfar * c->znear / depth);
    clip[i].x = ndc_x * z;
    clip[i].y = ndc_y * z;
    clip[i].z = clip_z;
    clip[i].w = z;
  }
}

/* K9 buildRenderVertices, K10 clear, K11 rasterTriangles (builtin_raster_renderer.cu:40-114),
 * K12 resolveRast (:119-172), K13 shadeRaster (raster_kernels.cuh:414-495), per hypothesis. */
void fpo_render(const float* verts, const float* normals, const float* colors, int nv,
                const int32_t* faces, int nf, const float* poses, const float* boxes, int batch,
                const float* k4, const fpo_config* c, float* out_rgb, float* out_xyz,
                float* out_rast) {
  const int W = c->input_width, H = c->input_height;
  const size_t P = (size_t)W * H;
  f4* clip = (f4*)malloc(sizeof(f4) * nv);
  f3* cp = (f3*)malloc(sizeof(f3) * nv);
  f3* cn = (f3*)malloc(sizeof(f3) * nv);
  uint64_t* zb = (uint64_t*)malloc(sizeof(uint64_t) * P);
  f4* rast = (f4*)malloc(sizeof(f4) * P);
  for (int s = 0; s < batch; ++s) {
    build_vertices(verts, normals, nv, poses + 16 * s, boxes + 4 * s, k4, c, clip, cp, cn);
    memset(zb, 0xFF, sizeof(uint64_t) * P);
    const float half_w = 0.5f * (float)W, half_h = 0.5f * (float)H;
    const float inv_w = 1.0f / (float)W, inv_h = 1.0f / (float)H;
    for (int tri = 0; tri < nf; ++tri) {
      const f4 p0 = clip[faces[3 * tri]], p1 = clip[faces[3 * tri + 1]], p2 = clip[faces[3 * tri + 2]];
      const float x0 = (p0.x / p0.w + 1.0f) * half_w - 0.5f;
      const float x1 = (p1.x / p1.w + 1.0f) * half_w - 0.5f;
      const float x2 = (p2.x / p2.w + 1.0f) * half_w - 0.5f;
      const float y0 = (p0.y / p0.w + 1.0f) * half_h - 0.5f;
      const float y1 = (p1.y / p1.w + 1.0f) * half_h - 0.5f;
      const float y2 = (p2.y / p2.w + 1.0f) * half_h - 0.5f;
      const int min_x = imax(0, (int)floorf(fminf(fminf(x0, x1), x2)));
      const int max_x = imin(W - 1, (int)ceilf(fmaxf(fmaxf(x0, x1), x2)));
      const int min_y = imax(0, (int)floorf(fminf(fminf(y0, y1), y2)));
      const int max_y = imin(H - 1, (int)ceilf(fmaxf(fmaxf(y0, y1), y2)));
      if (min_x > max_x || min_y > max_y) continue;
      for (int py = min_y; py <= max_y; ++py) {
        const float fy = (2.0f * py + 1.0f) * inv_h - 1.0f;
        const float p0y = p0.y - fy * p0.w, p1y = p1.y - fy * p1.w, p2y = p2.y - fy * p2.w;
        for (int px = min_x; px <= max_x; ++px) {
          const float fx = (2.0f * px + 1.0f) * inv_w - 1.0f;
          const float p0x = p0.x - fx * p0.w, p1x = p1.x - fx * p1.w, p2x = p2.x - fx * p2.w;
          const float a0 = p1x * p2y - p1y * p2x;
          const float a1 = p2x * p0y - p2y * p0x;
          const float a2 = p0x * p1y - p0y * p1x;
          const int inside_pos = a0 >= 0.0f && a1 >= 0.0f && a2 >= 0.0f;
          const int inside_neg = a0 <= 0.0f && a1 <= 0.0f && a2 <= 0.0f;
          const float area = a0 + a1 + a2;
          if ((!inside_pos && !inside_neg) || area == 0.0f) continue;
          const float z = p0.z * a0 + p1.z * a1 + p2.z * a2;
          const float wv = p0.w * a0 + p1.w * a1 + p2.w * a2;
          if (wv == 0.0f) continue;
          const uint64_t key = pack_depth_key(z / wv, tri + 1);
          uint64_t* slot = &zb[(size_t)py * W + px];
          if (key < *slot) *slot = key;
        }
      }
    }
    /* resolve */
    for (size_t lin = 0; lin < P; ++lin) {
      const uint64_t key = zb[lin];
      if (key == 0xFFFFFFFFFFFFFFFFull) {
        rast[lin].x = rast[lin].y = rast[lin].z = rast[lin].w = 0.0f;
        continue;
      }
      const int tp1 = (int)(key & 0xFFFFFFFFull);
      const int px = (int)(lin % W), py = (int)(lin / W);
      const f4 p0 = clip[faces[3 * (tp1 - 1)]], p1 = clip[faces[3 * (tp1 - 1) + 1]],
               p2 = clip[faces[3 * (tp1 - 1) + 2]];
      const float fx = (2.0f * px + 1.0f) / (float)W - 1.0f;
      const float fy = (2.0f * py + 1.0f) / (float)H - 1.0f;
      const float p0x = p0.x - fx * p0.w, p0y = p0.y - fy * p0.w;
      const float p1x = p1.x - fx * p1.w, p1y = p1.y - fy * p1.w;
      const float p2x = p2.x - fx * p2.w, p2y = p2.y - fy * p2.w;
      const float a0 = p1x * p2y - p1y * p2x;
      const float a1 = p2x * p0y - p2y * p0x;
      const float a2 = p0x * p1y - p0y * p1x;
      const float iw = 1.0f / (a0 + a1 + a2);
      float b0 = saturatef(a0 * iw), b1 = saturatef(a1 * iw);
      const float bs = 1.0f / fmaxf(b0 + b1, 1.0f);
      b0 *= bs;
      b1 *= bs;
      const float z = p0.z * a0 + p1.z * a1 + p2.z * a2;
      const float wv = p0.w * a0 + p1.w * a1 + p2.w * a2;
      const float zw = fmaxf(fminf(z / wv, 1.0f), -1.0f);
      rast[lin].x = b0;
      rast[lin].y = b1;
      rast[lin].z = zw;
      rast[lin].w = (float)tp1;
    }
    /* shade (rows flipped to top-down) */
    for (int y = 0; y < H; ++y)
      for (int x = 0; x < W; ++x) {
        const size_t o = ((size_t)s * H + y) * W + x;
        const f4 r = rast[(size_t)(H - 1 - y) * W + x];
        const int ti = (int)r.w - 1;
        float* rgb = out_rgb + 3 * o;
        float* xyz = out_xyz + 3 * o;
        if (ti < 0 || ti >= nf) {
          rgb[0] = rgb[1] = rgb[2] = xyz[0] = xyz[1] = xyz[2] = 0.0f;
          continue;
        }
        const int v0 = faces[3 * ti], v1 = faces[3 * ti + 1], v2 = faces[3 * ti + 2];
        const float b0 = r.x, b1 = r.y, b2 = fmaxf(0.0f, 1.0f - b0 - b1);
        const f3 q0 = cp[v0], q1 = cp[v1], q2 = cp[v2];
        xyz[0] = b0 * q0.x + b1 * q1.x + b2 * q2.x;
        xyz[1] = b0 * q0.y + b1 * q1.y + b2 * q2.y;
        xyz[2] = b0 * q0.z + b1 * q1.z + b2 * q2.z;
        const f3 n0 = cn[v0], n1 = cn[v1], n2 = cn[v2];
        const f3 n = normalize3(mk3(b0 * n0.x + b1 * n1.x + b2 * n2.x, b0 * n0.y + b1 * n1.y + b2 * n2.y,
                                    b0 * n0.z + b1 * n1.z + b2 * n2.z));
        const float* c0 = colors + 3 * v0;
        const float* c1 = colors + 3 * v1;
        const float* c2 = colors + 3 * v2;
        const float al[3] = {b0 * c0[0] + b1 * c1[0] + b2 * c2[0], b0 * c0[1] + b1 * c1[1] + b2 * c2[1],
                             b0 * c0[2] + b1 * c1[2] + b2 * c2[2]};
        const float diffuse = fmaxf(0.0f, -n.z);
        const float light = fminf(fmaxf(c->ambient_weight + c->diffuse_weight * diffuse, 0.0f), 1.5f);
        for (int ch = 0; ch < 3; ++ch) rgb[ch] = fminf(fmaxf(al[ch] * light, 0.0f), 1.0f);
      }
    if (out_rast) memcpy(out_rast + 4 * (size_t)s * P, rast, sizeof(f4) * P);
  }
  free(rast);
  free(zb);
  free(cn);
  free(cp);
  free(clip);
}

/* cuda_pipeline.cu:370-407 sampleRgbBilinear. */
static f3 sample_rgb_bilinear(const uint8_t* rgb, int w, int h, float x, float y) {
  if (x < 0.0f || y < 0.0f || x > (float)(w - 1) || y > (float)(h - 1)) return mk3(0, 0, 0);
  const int x0 = imin(imax((int)floorf(x), 0), w - 1);
  const int y0 = imin(imax((int)floorf(y), 0), h - 1);
  const int x1 = imin(x0 + 1, w - 1), y1 = imin(y0 + 1, h - 1);
  const float tx = x - (float)x0, ty = y - (float)y0;
  const uint8_t* q00 = rgb + (y0 * w + x0) * 3;
  const uint8_t* q10 = rgb + (y0 * w + x1) * 3;
  const uint8_t* q01 = rgb + (y1 * w + x0) * 3;
  const uint8_t* q11 = rgb + (y1 * w + x1) * 3;
  float o[3];
  for (int ch = 0; ch < 3; ++ch) {
    const float c00 = (float)q00[ch] / 255.0f, c10 = (float)q10[ch] / 255.0f;
    const float c01 = (float)q01[ch] / 255.0f, c11 = (float)q11[ch] / 255.0f;
    o[ch] = (1.0f - ty) * ((1.0f - tx) * c00 + tx * c10) + ty * ((1.0f - tx) * c01 + tx * c11);
  }
  return mk3(o[0], o[1], o[2]);
}

/* cuda_pipeline.cu:434-511 prepareNetworkInputsKernel. */
void fpo_pack(const uint8_t* rgb, const float* xyz_map, int img_w, int img_h,
              const float* rend_rgb, const float* rend_xyz, const float* poses,
              const float* boxes, int batch, int cw, int chh, float diameter, float thr,
              float* net_r, float* net_o) {
  const size_t P = (size_t)cw * chh;
  for (int s = 0; s < batch; ++s) {
    const float* box = boxes + 4 * s;
    const float crop_w = fmaxf(box[2] - box[0], 1.0f);
    const float crop_h = fmaxf(box[3] - box[1], 1.0f);
    const float* pose = poses + 16 * s;
    const f3 t = mk3(pose[3], pose[7], pose[11]);
    const float radius = fmaxf(diameter * 0.5f, 1e-6f);
    for (int y = 0; y < chh; ++y)
      for (int x = 0; x < cw; ++x) {
        float src_x = box[0] + (float)x * crop_w / (float)cw;
        float src_y = box[1] + (float)y * crop_h / (float)chh;
        if (img_w > 1) src_x = src_x * (float)img_w / (float)(img_w - 1) - 0.5f;
        if (img_h > 1) src_y = src_y * (float)img_h / (float)(img_h - 1) - 0.5f;
        const f3 orgb = sample_rgb_bilinear(rgb, img_w, img_h, src_x, src_y);
        f3 oxyz = mk3(0, 0, 0);
        const int xx = (int)roundf(src_x), yy = (int)roundf(src_y);
        if (!(xx < 0 || yy < 0 || xx >= img_w || yy >= img_h)) {
          const float* q = xyz_map + 3 * ((size_t)yy * img_w + xx);
          oxyz = mk3(q[0], q[1], q[2]);
        }
        const int obs_invalid = oxyz.z < thr;
        oxyz = mk3((oxyz.x - t.x) / radius, (oxyz.y - t.y) / radius, (oxyz.z - t.z) / radius);
        if (obs_invalid || fabsf(oxyz.x) >= 2.0f || fabsf(oxyz.y) >= 2.0f || fabsf(oxyz.z) >= 2.0f)
          oxyz = mk3(0, 0, 0);
        const size_t nhwc = ((size_t)s * chh + y) * cw + x;
        const float* rr = rend_rgb + 3 * nhwc;
        f3 rx = mk3(rend_xyz[3 * nhwc], rend_xyz[3 * nhwc + 1], rend_xyz[3 * nhwc + 2]);
        const int bg = rx.z < thr;
        rx = mk3((rx.x - t.x) / radius, (rx.y - t.y) / radius, (rx.z - t.z) / radius);
        if (bg) rx = mk3(0, 0, 0);
        const float rv[6] = {rr[0], rr[1], rr[2], rx.x, rx.y, rx.z};
        const float ov[6] = {orgb.x, orgb.y, orgb.z, oxyz.x, oxyz.y, oxyz.z};
        for (int ch = 0; ch < 6; ++ch) {
          net_r[((size_t)s * 6 + ch) * P + (size_t)y * cw + x] = rv[ch];
          net_o[((size_t)s * 6 + ch) * P + (size_t)y * cw + x] = ov[ch];
        }
      }
  }
}

/* cuda_pipeline.cu:46-85 so3ExpTranspose and :513-547 applyPoseDeltasKernel. */
void fpo_apply_deltas(float* poses, const float* dt, const float* dr, int batch, float diameter,
                      const fpo_config* c) {
  for (int i = 0; i < batch; ++i) {
    float* pose = poses + 16 * i;
    const float ox = tanhf(dr[3 * i + 0]) * c->rotation_normalizer_rad;
    const float oy = tanhf(dr[3 * i + 1]) * c->rotation_normalizer_rad;
    const float oz = tanhf(dr[3 * i + 2]) * c->rotation_normalizer_rad;
    float d[9] = {1, 0, 0, 0, 1, 0, 0, 0, 1};
    const float theta = sqrtf(fmaxf(ox * ox + oy * oy + oz * oz, 0.0f));
    if (!(theta < 1e-6f)) {
      const float inv = 1.0f / theta;
      const float x = ox * inv, y = oy * inv, z = oz * inv;
      const float s = sinf(theta), cth = cosf(theta), oc = 1.0f - cth;
      const float r[9] = {cth + x * x * oc,     x * y * oc - z * s, x * z * oc + y * s,
                          y * x * oc + z * s,   cth + y * y * oc,   y * z * oc - x * s,
                          z * x * oc - y * s,   z * y * oc + x * s, cth + z * z * oc};
      mat3_transpose(r, d);
    }
    const float old_r[9] = {pose[0], pose[1], pose[2], pose[4], pose[5], pose[6], pose[8], pose[9], pose[10]};
    for (int row = 0; row < 3; ++row)
      for (int col = 0; col < 3; ++col) {
        float v = 0.0f;
        for (int k = 0; k < 3; ++k) v += d[row * 3 + k] * old_r[k * 3 + col];
        pose[row * 4 + col] = v;
      }
    const float scale = diameter * 0.5f;
    pose[3] += dt[3 * i + 0] * scale;
    pose[7] += dt[3 * i + 1] * scale;
    pose[11] += dt[3 * i + 2] * scale;
  }
}

/* cuda_pipeline.cu:549-582 selectBestPoseKernel (strict '>', first max wins). */
int fpo_select_best(const float* poses, const float* scores, int batch, const float* center,
                    float* out, float* out_score) {
  int best = 0;
  float best_score = scores[0];
  for (int i = 1; i < batch; ++i)
    if (scores[i] > best_score) {
      best_score = scores[i];
      best = i;
    }
  const float* src = poses + 16 * best;
  for (int i = 0; i < 16; ++i) out[i] = 0.0f;
  out[15] = 1.0f;
  for (int r = 0; r < 3; ++r)
    for (int cc = 0; cc < 3; ++cc) out[r * 4 + cc] = src[r * 4 + cc];
  const float nc[3] = {-center[0], -center[1], -center[2]};
  for (int r = 0; r < 3; ++r)
    out[r * 4 + 3] = src[r * 4 + 3] + src[r * 4 + 0] * nc[0] + src[r * 4 + 1] * nc[1] + src[r * 4 + 2] * nc[2];
  *out_score = best_score;
  return best;
}

/* mesh.cpp:589-610 computeVertexNormals. */
void fpo_vertex_normals(const float* verts, int nv, const int32_t* faces, int nf, float* normals) {
  f3* acc = (f3*)calloc((size_t)nv, sizeof(f3));
  for (int i = 0; i < nf; ++i) {
    const int ia = faces[3 * i], ib = faces[3 * i + 1], ic = faces[3 * i + 2];
    if (ia < 0 || ib < 0 || ic < 0 || ia >= nv || ib >= nv || ic >= nv) continue;
    const f3 a = mk3(verts[3 * ia], verts[3 * ia + 1], verts[3 * ia + 2]);
    const f3 b = mk3(verts[3 * ib], verts[3 * ib + 1], verts[3 * ib + 2]);
    const f3 cc = mk3(verts[3 * ic], verts[3 * ic + 1], verts[3 * ic + 2]);
    const f3 n = cross3(mk3(b.x - a.x, b.y - a.y, b.z - a.z), mk3(cc.x - a.x, cc.y - a.y, cc.z - a.z));
    const int id[3] = {ia, ib, ic};
    for (int k = 0; k < 3; ++k) {
      acc[id[k]].x = acc[id[k]].x + n.x;
      acc[id[k]].y = acc[id[k]].y + n.y;
      acc[id[k]].z = acc[id[k]].z + n.z;
    }
  }
  for (int i = 0; i < nv; ++i) {
    f3 n = normalize_host(acc[i]);
    if (norm3(n) < 1e-6f) n = mk3(0.0f, 0.0f, 1.0f);
    normals[3 * i] = n.x;
    normals[3 * i + 1] = n.y;
    normals[3 * i + 2] = n.z;
  }
  free(acc);
}

/* mesh.cpp:612-660 preprocessMesh: bbox centre, strided-sample O(n^2) diameter. */
void fpo_mesh_center_diameter(const float* verts, int nv, int sample_points, float* center,
                              float* diameter, float* centered) {
  f3 mn = mk3(FLT_MAX, FLT_MAX, FLT_MAX), mx = mk3(-FLT_MAX, -FLT_MAX, -FLT_MAX);
  for (int i = 0; i < nv; ++i) {
    mn.x = fminf(mn.x, verts[3 * i]);
    mn.y = fminf(mn.y, verts[3 * i + 1]);
    mn.z = fminf(mn.z, verts[3 * i + 2]);
    mx.x = fmaxf(mx.x, verts[3 * i]);
    mx.y = fmaxf(mx.y, verts[3 * i + 1]);
    mx.z = fmaxf(mx.z, verts[3 * i + 2]);
  }
  const f3 ctr = mk3((mn.x + mx.x) * 0.5f, (mn.y + mx.y) * 0.5f, (mn.z + mx.z) * 0.5f);
  center[0] = ctr.x;
  center[1] = ctr.y;
  center[2] = ctr.z;
  for (int i = 0; i < nv; ++i) {
    centered[3 * i] = verts[3 * i] - ctr.x;
    centered[3 * i + 1] = verts[3 * i + 1] - ctr.y;
    centered[3 * i + 2] = verts[3 * i + 2] - ctr.z;
  }
  const size_t sample_count = (size_t)imin(sample_points, nv);
  size_t stride = (size_t)nv / sample_count;
  if (stride < 1) stride = 1;
  f3* s = (f3*)malloc(sizeof(f3) * sample_count);
  size_t ns = 0;
  for (size_t i = 0; i < (size_t)nv && ns < sample_count; i += stride)
    s[ns++] = mk3(centered[3 * i], centered[3 * i + 1], centered[3 * i + 2]);
  float d = 0.0f;
  for (size_t i = 0; i < ns; ++i)
    for (size_t j = i + 1; j < ns; ++j)
      d = fmaxf(d, norm3(mk3(s[i].x - s[j].x, s[i].y - s[j].y, s[i].z - s[j].z)));
  free(s);
  if (d <= 0.0f) d = norm3(mk3(mx.x - mn.x, mx.y - mn.y, mx.z - mn.z));
  *diameter = fmaxf(d, 1e-6f);
}
