// Triangle rasterizer for candidate-scene previews (CUDA) with a CPU restatement of the same math.
//
// The reference renders three.js scenes through WebGL on SwiftShader in headless Chrome
// (pipeline_service/modules/renderer/render_service/object-page.html:202-274). There is no graphics
// stack here, so scenes are flattened to world-space triangles and drawn by:
//   pass 1 (one thread per triangle): project the vertices with the 4x4 view-projection matrix, clip
//     triangles behind the camera, walk the screen bounding box with edge functions (pixel centres,
//     top-left fill), interpolate depth, and keep the nearest (depth, triangle id) per pixel with a 64-bit
//     atomicMin on (float depth bits << 32 | id) — deterministic: ties go to the lower triangle id;
//   pass 2 (one thread per pixel): shade the winning triangle: two-sided Lambert from a directional light
//     plus ambient, ACES filmic tone map (Narkowicz's rational fit), sRGB encoding, 8-bit RGBA.
// raster_pbr shades like a metallic-roughness standard material instead: up to four directional lights
// (fixed directions, or following the camera) with a GGX specular lobe -- Trowbridge-Reitz distribution,
// height-correlated Smith visibility, Schlick Fresnel with F0 = mix(0.04, albedo, metalness) -- plus a
// Lambert term of (1 - metalness) x albedo, an ambient term, and a hemisphere environment (sky / ground
// colours blended by the normal's, and for the specular the reflection's, height) whose specular response
// uses Karis' analytic split-sum approximation ("Physically Based Shading on Mobile", 2014). The reference
// lights its pages with a PMREM environment plus directional, hemisphere and camera-follow lights on
// MeshStandardMaterial (render_service/object-page.html:33-120); this is a closed-form restatement of that
// kind of rig, not a reproduction of WebGL's output.
// The CPU branch of each entry point runs the identical code on the host and is the oracle of the GPU path.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cmath>
#include <cstring>

namespace phx {

struct RasterParams {
  int W, H, T;
  float vp[16];        // row-major view-projection
  float light[3];      // direction towards the light (normalised)
  float ambient, diffuse, exposure;
  float bg[3];         // linear background colour
};

__host__ __device__ inline void project(const RasterParams& p, const float* v, float& sx, float& sy, float& z, float& w) {
  const float x = v[0], y = v[1], zz = v[2];
  const float cx = p.vp[0] * x + p.vp[1] * y + p.vp[2] * zz + p.vp[3];
  const float cy = p.vp[4] * x + p.vp[5] * y + p.vp[6] * zz + p.vp[7];
  const float cz = p.vp[8] * x + p.vp[9] * y + p.vp[10] * zz + p.vp[11];
  w = p.vp[12] * x + p.vp[13] * y + p.vp[14] * zz + p.vp[15];
  const float iw = 1.0f / w;
  sx = (cx * iw * 0.5f + 0.5f) * p.W;
  sy = (1.0f - (cy * iw * 0.5f + 0.5f)) * p.H;
  z = cz * iw;
}

__host__ __device__ inline float edge(float ax, float ay, float bx, float by, float px, float py) {
  return (bx - ax) * (py - ay) - (by - ay) * (px - ax);
}

__host__ __device__ inline unsigned long long pack_depth(float z, int id) {
  unsigned int zb;
  memcpy(&zb, &z, 4);  // z in [0, 1] (non-negative): float order == unsigned order
  return (static_cast<unsigned long long>(zb) << 32) | static_cast<unsigned int>(id);
}

// visit the covered pixels of triangle t; fn(pixel_index, depth)
template <typename F>
__host__ __device__ inline void raster_triangle(const RasterParams& p, const float* tri, F fn) {
  float x[3], y[3], z[3], w[3];
  for (int i = 0; i < 3; ++i) project(p, tri + 3 * i, x[i], y[i], z[i], w[i]);
  if (w[0] <= 1e-6f || w[1] <= 1e-6f || w[2] <= 1e-6f) return;   // behind the camera (no clipping)
  float area = edge(x[0], y[0], x[1], y[1], x[2], y[2]);
  if (fabsf(area) < 1e-12f) return;
  if (area < 0) {  // two-sided: make the winding counter-clockwise in screen space
    float tx = x[1], ty = y[1], tz = z[1];
    x[1] = x[2], y[1] = y[2], z[1] = z[2];
    x[2] = tx, y[2] = ty, z[2] = tz;
    area = -area;
  }
  int x0 = (int)floorf(fminf(x[0], fminf(x[1], x[2])));
  int x1 = (int)ceilf(fmaxf(x[0], fmaxf(x[1], x[2])));
  int y0 = (int)floorf(fminf(y[0], fminf(y[1], y[2])));
  int y1 = (int)ceilf(fmaxf(y[0], fmaxf(y[1], y[2])));
  x0 = x0 < 0 ? 0 : x0;
  y0 = y0 < 0 ? 0 : y0;
  x1 = x1 > p.W - 1 ? p.W - 1 : x1;
  y1 = y1 > p.H - 1 ? p.H - 1 : y1;
  const float ia = 1.0f / area;
  for (int py = y0; py <= y1; ++py) {
    for (int px = x0; px <= x1; ++px) {
      const float cx = px + 0.5f, cy = py + 0.5f;
      const float w0 = edge(x[1], y[1], x[2], y[2], cx, cy);
      const float w1 = edge(x[2], y[2], x[0], y[0], cx, cy);
      const float w2 = edge(x[0], y[0], x[1], y[1], cx, cy);
      if (w0 < 0 || w1 < 0 || w2 < 0) continue;
      const float d = (w0 * z[0] + w1 * z[1] + w2 * z[2]) * ia;
      if (d < 0.f || d > 1.f) continue;
      fn(py * p.W + px, d);
    }
  }
}

__host__ __device__ inline float aces(float x) {
  const float a = 2.51f, b = 0.03f, c = 2.43f, d = 0.59f, e = 0.14f;
  const float y = (x * (a * x + b)) / (x * (c * x + d) + e);
  return y < 0.f ? 0.f : (y > 1.f ? 1.f : y);
}

__host__ __device__ inline float srgb(float x) {
  return x <= 0.0031308f ? 12.92f * x : 1.055f * powf(x, 1.0f / 2.4f) - 0.055f;
}

__host__ __device__ inline void shade(const RasterParams& p, const float* tri, const float* col, unsigned char* out) {
  const float e1[3] = {tri[3] - tri[0], tri[4] - tri[1], tri[5] - tri[2]};
  const float e2[3] = {tri[6] - tri[0], tri[7] - tri[1], tri[8] - tri[2]};
  float n[3] = {e1[1] * e2[2] - e1[2] * e2[1], e1[2] * e2[0] - e1[0] * e2[2], e1[0] * e2[1] - e1[1] * e2[0]};
  const float len = sqrtf(n[0] * n[0] + n[1] * n[1] + n[2] * n[2]);
  const float ndl = len > 0.f ? fabsf(n[0] * p.light[0] + n[1] * p.light[1] + n[2] * p.light[2]) / len : 0.f;
  const float k = p.ambient + p.diffuse * ndl;
  for (int c = 0; c < 3; ++c) {
    const float v = srgb(aces(col[c] * k * p.exposure));
    int q = (int)(v * 255.0f + 0.5f);
    out[c] = (unsigned char)(q < 0 ? 0 : (q > 255 ? 255 : q));
  }
  out[3] = 255;
}

__host__ __device__ inline void shade_bg(const RasterParams& p, unsigned char* out) {
  for (int c = 0; c < 3; ++c) {
    const float v = srgb(p.bg[c] < 0.f ? 0.f : (p.bg[c] > 1.f ? 1.f : p.bg[c]));
    int q = (int)(v * 255.0f + 0.5f);
    out[c] = (unsigned char)(q < 0 ? 0 : (q > 255 ? 255 : q));
  }
  out[3] = 255;
}

// ------------------------------------------------------------------------------------------------
// standard-material shading
// ------------------------------------------------------------------------------------------------
struct PbrParams {
  float eye[3];
  int nl;
  float ldir[4][3];    // direction towards each light (normalised); ignored for camera-follow lights
  float lint[4];
  int lfollow[4];
  float ambient;
  float sky[3], ground[3], env;   // hemisphere environment (linear colours) and its intensity
};

__host__ __device__ inline float dot3(const float* a, const float* b) { return a[0] * b[0] + a[1] * b[1] + a[2] * b[2]; }
__host__ __device__ inline void norm3(float* a) {
  const float l = sqrtf(dot3(a, a));
  if (l > 0.f) a[0] /= l, a[1] /= l, a[2] /= l;
}

__host__ __device__ inline void shade_pbr(const RasterParams& p, const PbrParams& q, const float* tri, const float* col,
                                          const float* mat, unsigned char* out) {
  const float e1[3] = {tri[3] - tri[0], tri[4] - tri[1], tri[5] - tri[2]};
  const float e2[3] = {tri[6] - tri[0], tri[7] - tri[1], tri[8] - tri[2]};
  float n[3] = {e1[1] * e2[2] - e1[2] * e2[1], e1[2] * e2[0] - e1[0] * e2[2], e1[0] * e2[1] - e1[1] * e2[0]};
  norm3(n);
  float v[3] = {q.eye[0] - (tri[0] + tri[3] + tri[6]) / 3.f, q.eye[1] - (tri[1] + tri[4] + tri[7]) / 3.f,
                q.eye[2] - (tri[2] + tri[5] + tri[8]) / 3.f};
  norm3(v);
  if (dot3(n, v) < 0.f) n[0] = -n[0], n[1] = -n[1], n[2] = -n[2];   // two-sided
  const float rough = fminf(fmaxf(mat ? mat[0] : 1.f, 0.04f), 1.f);
  const float metal = fminf(fmaxf(mat ? mat[1] : 0.f, 0.f), 1.f);
  const float a = rough * rough, a2 = a * a;
  const float ndv = fmaxf(dot3(n, v), 1e-4f);
  const float kPi = 3.14159265358979f;
  float f0[3], kd[3], lo[3] = {0.f, 0.f, 0.f};
  for (int c = 0; c < 3; ++c) {
    f0[c] = 0.04f * (1.f - metal) + col[c] * metal;
    kd[c] = col[c] * (1.f - metal);
  }
  for (int i = 0; i < q.nl && i < 4; ++i) {
    float l[3] = {q.ldir[i][0], q.ldir[i][1], q.ldir[i][2]};
    if (q.lfollow[i]) l[0] = v[0], l[1] = v[1], l[2] = v[2];
    const float ndl = dot3(n, l);
    if (ndl <= 0.f) continue;
    float h[3] = {l[0] + v[0], l[1] + v[1], l[2] + v[2]};
    norm3(h);
    const float ndh = fmaxf(dot3(n, h), 0.f), vdh = fmaxf(dot3(v, h), 0.f);
    const float dd = ndh * ndh * (a2 - 1.f) + 1.f;
    const float D = a2 / (kPi * dd * dd);
    const float vis = 0.5f / (ndl * sqrtf(ndv * ndv * (1.f - a2) + a2) + ndv * sqrtf(ndl * ndl * (1.f - a2) + a2));
    const float fw = powf(1.f - vdh, 5.f);
    for (int c = 0; c < 3; ++c) {
      const float F = f0[c] + (1.f - f0[c]) * fw;
      lo[c] += q.lint[i] * ndl * (kd[c] / kPi + D * vis * F);
    }
  }
  // environment: hemisphere irradiance for the diffuse term, the reflection direction's colour for the specular
  const float r[3] = {2.f * ndv * n[0] - v[0], 2.f * ndv * n[1] - v[1], 2.f * ndv * n[2] - v[2]};
  const float wd = 0.5f + 0.5f * n[1], ws = 0.5f + 0.5f * r[1];
  // Karis 2014 analytic environment BRDF: (A, B) scale and bias of F0
  const float c0x = -1.f, c0y = -0.0275f, c0z = -0.572f, c0w = 0.022f;
  const float c1x = 1.f, c1y = 0.0425f, c1z = 1.04f, c1w = -0.04f;
  const float rx = rough * c0x + c1x, ry = rough * c0y + c1y, rz = rough * c0z + c1z, rw = rough * c0w + c1w;
  const float a004 = fminf(rx * rx, exp2f(-9.28f * ndv)) * rx + ry;
  const float A = -1.04f * a004 + rz, B = 1.04f * a004 + rw;
  for (int c = 0; c < 3; ++c) {
    const float irr = q.ground[c] + (q.sky[c] - q.ground[c]) * wd;
    const float rad = q.ground[c] + (q.sky[c] - q.ground[c]) * ws;
    lo[c] += q.env * (irr * kd[c] + rad * (f0[c] * A + B)) + q.ambient * kd[c] / kPi;
  }
  for (int c = 0; c < 3; ++c) {
    const float x = srgb(aces(lo[c] * p.exposure));
    int qv = (int)(x * 255.0f + 0.5f);
    out[c] = (unsigned char)(qv < 0 ? 0 : (qv > 255 ? 255 : qv));
  }
  out[3] = 255;
}

__global__ void raster_pass1(const RasterParams p, const float* __restrict__ tris, unsigned long long* __restrict__ zbuf) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= p.T) return;
  raster_triangle(p, tris + 9 * t, [&](int pix, float d) { atomicMin(zbuf + pix, pack_depth(d, t)); });
}

__global__ void raster_pass2(const RasterParams p, const float* __restrict__ tris, const float* __restrict__ cols,
                             const unsigned long long* __restrict__ zbuf, unsigned char* __restrict__ img) {
  const int pix = blockIdx.x * blockDim.x + threadIdx.x;
  if (pix >= p.W * p.H) return;
  const unsigned long long z = zbuf[pix];
  if (z == ~0ull) {
    shade_bg(p, img + 4 * pix);
    return;
  }
  const int t = (int)(z & 0xffffffffull);
  shade(p, tris + 9 * t, cols + 3 * t, img + 4 * pix);
}

__global__ void raster_pass2_pbr(const RasterParams p, const PbrParams q, const float* __restrict__ tris,
                                 const float* __restrict__ cols, const float* __restrict__ mats,
                                 const unsigned long long* __restrict__ zbuf, unsigned char* __restrict__ img) {
  const int pix = blockIdx.x * blockDim.x + threadIdx.x;
  if (pix >= p.W * p.H) return;
  const unsigned long long z = zbuf[pix];
  if (z == ~0ull) {
    shade_bg(p, img + 4 * pix);
    return;
  }
  const int t = (int)(z & 0xffffffffull);
  shade_pbr(p, q, tris + 9 * t, cols + 3 * t, mats ? mats + 2 * t : nullptr, img + 4 * pix);
}

static RasterParams make_params(int W, int H, int T, torch::Tensor vp, std::vector<double> light, double ambient,
                                double diffuse, double exposure, std::vector<double> bg) {
  TORCH_CHECK(vp.numel() == 16 && light.size() == 3 && bg.size() == 3);
  RasterParams p;
  p.W = W, p.H = H, p.T = T;
  auto v = vp.to(torch::kCPU, torch::kFloat).contiguous();
  for (int i = 0; i < 16; ++i) p.vp[i] = v.data_ptr<float>()[i];
  const double ln = std::sqrt(light[0] * light[0] + light[1] * light[1] + light[2] * light[2]);
  for (int i = 0; i < 3; ++i) p.light[i] = (float)(light[i] / (ln > 0 ? ln : 1.0)), p.bg[i] = (float)bg[i];
  p.ambient = (float)ambient, p.diffuse = (float)diffuse, p.exposure = (float)exposure;
  return p;
}

torch::Tensor raster(torch::Tensor tris, torch::Tensor cols, torch::Tensor vp, int64_t W, int64_t H,
                     std::vector<double> light, double ambient, double diffuse, double exposure, std::vector<double> bg) {
  TORCH_CHECK(tris.scalar_type() == at::kFloat && tris.dim() == 3 && tris.size(1) == 3 && tris.size(2) == 3);
  TORCH_CHECK(cols.scalar_type() == at::kFloat && cols.size(0) == tris.size(0) && cols.size(1) == 3);
  tris = tris.contiguous();
  cols = cols.contiguous();
  const int T = tris.size(0);
  const RasterParams p = make_params((int)W, (int)H, T, vp, light, ambient, diffuse, exposure, bg);
  auto img = torch::empty({H, W, 4}, tris.options().dtype(at::kByte));
  if (!tris.is_cuda()) {  // CPU oracle: same algorithm, sequential
    std::vector<unsigned long long> zb((size_t)W * H, ~0ull);
    const float* tp = tris.data_ptr<float>();
    for (int t = 0; t < T; ++t)
      raster_triangle(p, tp + 9 * t, [&](int pix, float d) {
        const unsigned long long v = pack_depth(d, t);
        if (v < zb[pix]) zb[pix] = v;
      });
    unsigned char* o = img.data_ptr<unsigned char>();
    const float* cp = cols.data_ptr<float>();
    for (int pix = 0; pix < W * H; ++pix) {
      if (zb[pix] == ~0ull)
        shade_bg(p, o + 4 * pix);
      else {
        const int t = (int)(zb[pix] & 0xffffffffull);
        shade(p, tp + 9 * t, cp + 3 * t, o + 4 * pix);
      }
    }
    return img;
  }
  const at::cuda::CUDAGuard guard(tris.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  auto zbuf = torch::empty({H * W}, tris.options().dtype(at::kLong));
  cudaMemsetAsync(zbuf.data_ptr(), 0xff, (size_t)H * W * 8, stream);
  if (T > 0)
    raster_pass1<<<(T + 127) / 128, 128, 0, stream>>>(p, tris.data_ptr<float>(),
                                                       reinterpret_cast<unsigned long long*>(zbuf.data_ptr()));
  raster_pass2<<<(int)((W * H + 255) / 256), 256, 0, stream>>>(p, tris.data_ptr<float>(), cols.data_ptr<float>(),
                                                                reinterpret_cast<unsigned long long*>(zbuf.data_ptr()),
                                                                img.data_ptr<unsigned char>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return img;
}

// Standard-material variant. lights: [L, 5] rows (dx, dy, dz, intensity, follow) with L <= 4 (follow != 0: the
// light sits at the camera); hemi: (sky rgb, ground rgb, intensity) linear; mats: [T, 2] (roughness, metalness)
// or empty (roughness 1, metalness 0, the standard material's defaults).
torch::Tensor raster_pbr(torch::Tensor tris, torch::Tensor cols, torch::Tensor mats, torch::Tensor vp,
                         std::vector<double> eye, torch::Tensor lights, double ambient, std::vector<double> hemi,
                         double exposure, std::vector<double> bg, int64_t W, int64_t H) {
  TORCH_CHECK(tris.scalar_type() == at::kFloat && tris.dim() == 3 && tris.size(1) == 3 && tris.size(2) == 3);
  TORCH_CHECK(cols.scalar_type() == at::kFloat && cols.size(0) == tris.size(0) && cols.size(1) == 3);
  TORCH_CHECK(eye.size() == 3 && hemi.size() == 7);
  const bool has_mat = mats.numel() > 0;
  if (has_mat) TORCH_CHECK(mats.scalar_type() == at::kFloat && mats.size(0) == tris.size(0) && mats.size(1) == 2);
  tris = tris.contiguous();
  cols = cols.contiguous();
  if (has_mat) mats = mats.contiguous();
  const int T = tris.size(0);
  const RasterParams p = make_params((int)W, (int)H, T, vp, {0.0, 1.0, 0.0}, 0.0, 0.0, exposure, bg);
  PbrParams q{};
  for (int i = 0; i < 3; ++i) q.eye[i] = (float)eye[i], q.sky[i] = (float)hemi[i], q.ground[i] = (float)hemi[3 + i];
  q.env = (float)hemi[6];
  q.ambient = (float)ambient;
  auto lc = lights.to(torch::kCPU, torch::kFloat).contiguous();
  TORCH_CHECK(lc.dim() == 2 && lc.size(1) == 5 && lc.size(0) <= 4, "lights: [L <= 4, 5]");
  q.nl = (int)lc.size(0);
  for (int i = 0; i < q.nl; ++i) {
    const float* r = lc.data_ptr<float>() + 5 * i;
    float d[3] = {r[0], r[1], r[2]};
    norm3(d);
    for (int c = 0; c < 3; ++c) q.ldir[i][c] = d[c];
    q.lint[i] = r[3];
    q.lfollow[i] = r[4] != 0.f;
  }
  auto img = torch::empty({H, W, 4}, tris.options().dtype(at::kByte));
  if (!tris.is_cuda()) {
    std::vector<unsigned long long> zb((size_t)W * H, ~0ull);
    const float* tp = tris.data_ptr<float>();
    for (int t = 0; t < T; ++t)
      raster_triangle(p, tp + 9 * t, [&](int pix, float d) {
        const unsigned long long v = pack_depth(d, t);
        if (v < zb[pix]) zb[pix] = v;
      });
    unsigned char* o = img.data_ptr<unsigned char>();
    const float* cp = cols.data_ptr<float>();
    const float* mp = has_mat ? mats.data_ptr<float>() : nullptr;
    for (int pix = 0; pix < W * H; ++pix) {
      if (zb[pix] == ~0ull)
        shade_bg(p, o + 4 * pix);
      else {
        const int t = (int)(zb[pix] & 0xffffffffull);
        shade_pbr(p, q, tp + 9 * t, cp + 3 * t, mp ? mp + 2 * t : nullptr, o + 4 * pix);
      }
    }
    return img;
  }
  const at::cuda::CUDAGuard guard(tris.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  auto zbuf = torch::empty({H * W}, tris.options().dtype(at::kLong));
  cudaMemsetAsync(zbuf.data_ptr(), 0xff, (size_t)H * W * 8, stream);
  if (T > 0)
    raster_pass1<<<(T + 127) / 128, 128, 0, stream>>>(p, tris.data_ptr<float>(),
                                                       reinterpret_cast<unsigned long long*>(zbuf.data_ptr()));
  raster_pass2_pbr<<<(int)((W * H + 255) / 256), 256, 0, stream>>>(
      p, q, tris.data_ptr<float>(), cols.data_ptr<float>(), has_mat ? mats.data_ptr<float>() : nullptr,
      reinterpret_cast<unsigned long long*>(zbuf.data_ptr()), img.data_ptr<unsigned char>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return img;
}

}  // namespace phx
