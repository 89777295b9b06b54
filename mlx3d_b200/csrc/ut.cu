// Unscented-transform projection (3DGUT; src/mlx3d/splatting/projection.py:
// 149-205): six sigma points mean +- sqrt(3) * (column k of R(q) diag(s))
// through the camera's own projection (cameras.py:290-317: orthographic,
// pinhole, Brown-Conrady or fisheye distortion), their sample mean and
// covariance give means2d and the blurred 2-D covariance; conic,
// compensation and radius follow as in the EWA projection.  One thread per
// Gaussian; forward in the reference's float32 operation order (exactly
// rounded primitives), backward hand-derived.
#include "gs_common.cuh"

namespace gs {

struct UtArgs {
  gs_camera cam;
  gs_lens lens;
  const float *means, *quats, *scales;
  int64_t n;
  float blur;
  int aa;
  float *means2d, *conics, *depths, *radii, *comp;
  // backward
  const float *g_means2d, *g_conics, *g_depths, *g_comp;
  float *g_means, *g_quats, *g_scales;
};

__device__ __forceinline__ void quat_rot(const float* q, float* w4, float R[3][3]) {
  const float nrm = gs_sqrt(gs_add(gs_add(gs_add(gs_mul(q[0], q[0]), gs_mul(q[1], q[1])), gs_mul(q[2], q[2])), gs_mul(q[3], q[3])));
  const float w = gs_div(q[0], nrm), x = gs_div(q[1], nrm), y = gs_div(q[2], nrm), z = gs_div(q[3], nrm);
  w4[0] = w; w4[1] = x; w4[2] = y; w4[3] = z;
  R[0][0] = gs_sub(1.0f, gs_mul(2.0f, gs_add(gs_mul(y, y), gs_mul(z, z))));
  R[0][1] = gs_mul(2.0f, gs_sub(gs_mul(x, y), gs_mul(w, z)));
  R[0][2] = gs_mul(2.0f, gs_add(gs_mul(x, z), gs_mul(w, y)));
  R[1][0] = gs_mul(2.0f, gs_add(gs_mul(x, y), gs_mul(w, z)));
  R[1][1] = gs_sub(1.0f, gs_mul(2.0f, gs_add(gs_mul(x, x), gs_mul(z, z))));
  R[1][2] = gs_mul(2.0f, gs_sub(gs_mul(y, z), gs_mul(w, x)));
  R[2][0] = gs_mul(2.0f, gs_sub(gs_mul(x, z), gs_mul(w, y)));
  R[2][1] = gs_mul(2.0f, gs_add(gs_mul(y, z), gs_mul(w, x)));
  R[2][2] = gs_sub(1.0f, gs_mul(2.0f, gs_add(gs_mul(x, x), gs_mul(y, y))));
}

// world -> camera (points @ R^T + t), one row.
__device__ __forceinline__ float cam_row(const gs_camera& c, int i, float p0, float p1, float p2) {
  return gs_add(gs_add(gs_add(gs_mul(p0, c.R[3 * i]), gs_mul(p1, c.R[3 * i + 1])), gs_mul(p2, c.R[3 * i + 2])), c.t[i]);
}

// Camera.project_points for one world point (cameras.py:290-317, distortion
// :42-50 and :68-76); optionally its 2x3 Jacobian d(u, v)/d(point).
__device__ __forceinline__ void project_point(const gs_camera& c, const gs_lens& L, float p0, float p1, float p2,
                                              float& u, float& v, float J[2][3]) {
  const float pcx = cam_row(c, 0, p0, p1, p2), pcy = cam_row(c, 1, p0, p1, p2), z = cam_row(c, 2, p0, p1, p2);
  float du_dpc[2][3];
  if (L.orthographic) {
    u = gs_add(gs_mul(c.fx, pcx), c.cx);
    v = gs_add(gs_mul(c.fy, pcy), c.cy);
    du_dpc[0][0] = c.fx; du_dpc[0][1] = 0.f; du_dpc[0][2] = 0.f;
    du_dpc[1][0] = 0.f; du_dpc[1][1] = c.fy; du_dpc[1][2] = 0.f;
  } else {
    const float eps = 1e-8f;
    const bool clamped = fabsf(z) < eps;
    const float zz = clamped ? eps : z;
    const float inv = gs_div(1.0f, zz);
    const float x = gs_mul(pcx, inv), y = gs_mul(pcy, inv);
    // d(x, y) / d(pcx, pcy, z)
    const float dxz = clamped ? 0.f : -x * inv, dyz = clamped ? 0.f : -y * inv;
    float xd = x, yd = y, a = 1.f, b = 0.f, cc = 0.f, d = 1.f;  // d(xd, yd)/d(x, y) = [[a, b], [cc, d]]
    if (L.n_dist > 0 && !L.fisheye) {
      const float k1 = L.dist[0], k2 = L.dist[1], p1 = L.dist[2], p2 = L.dist[3], k3 = L.dist[4];
      const float r2 = gs_add(gs_mul(x, x), gs_mul(y, y));
      const float radial = gs_add(1.0f, gs_mul(r2, gs_add(k1, gs_mul(r2, gs_add(k2, gs_mul(r2, k3))))));
      const float p1x2 = L.dist[2] * 2.0f, p2x2 = L.dist[3] * 2.0f;  // float(2.0 * p) (exact doubling)
      xd = gs_add(gs_add(gs_mul(x, radial), gs_mul(gs_mul(p1x2, x), y)),
                  gs_mul(p2, gs_add(r2, gs_mul(gs_mul(2.0f, x), x))));
      yd = gs_add(gs_add(gs_mul(y, radial), gs_mul(p1, gs_add(r2, gs_mul(gs_mul(2.0f, y), y)))),
                  gs_mul(gs_mul(p2x2, x), y));
      const float dR = k1 + 2.f * k2 * r2 + 3.f * k3 * r2 * r2;
      a = radial + 2.f * x * x * dR + 2.f * p1 * y + 6.f * p2 * x;
      b = 2.f * x * y * dR + 2.f * p1 * x + 2.f * p2 * y;
      cc = 2.f * x * y * dR + 2.f * p1 * x + 2.f * p2 * y;
      d = radial + 2.f * y * y * dR + 6.f * p1 * y + 2.f * p2 * x;
    } else if (L.n_dist > 0) {
      const float k1 = L.dist[0], k2 = L.dist[1], k3 = L.dist[2], k4 = L.dist[3];
      const float r = gs_sqrt(gs_add(gs_mul(x, x), gs_mul(y, y)));
      const float th = atanf(r);
      const float t2 = gs_mul(th, th);
      const float thd = gs_mul(th, gs_add(1.0f, gs_mul(t2, gs_add(k1, gs_mul(t2, gs_add(k2, gs_mul(t2, gs_add(k3, gs_mul(t2, k4)))))))));
      const float epsf = 1e-9f;
      const float rs = gs_maxf(r, epsf);
      const float sc = gs_div(thd, rs);
      xd = gs_mul(x, sc);
      yd = gs_mul(y, sc);
      const float dthd = 1.f + t2 * (3.f * k1 + t2 * (5.f * k2 + t2 * (7.f * k3 + t2 * 9.f * k4)));
      const float dth_dr = 1.f / (1.f + r * r);
      const float dsc_dr = r > epsf ? (dthd * dth_dr * r - thd) / (r * r) : dthd * dth_dr / epsf;
      const float rx = r > 0.f ? x / r : 0.f, ry = r > 0.f ? y / r : 0.f;
      a = sc + x * dsc_dr * rx;
      b = x * dsc_dr * ry;
      cc = y * dsc_dr * rx;
      d = sc + y * dsc_dr * ry;
    }
    u = gs_add(gs_mul(c.fx, xd), c.cx);
    v = gs_add(gs_mul(c.fy, yd), c.cy);
    // chain: (u, v) <- (xd, yd) <- (x, y) <- (pcx, pcy, z)
    const float dx[3] = {inv, 0.f, dxz}, dy[3] = {0.f, inv, dyz};
    for (int k = 0; k < 3; ++k) {
      du_dpc[0][k] = c.fx * (a * dx[k] + b * dy[k]);
      du_dpc[1][k] = c.fy * (cc * dx[k] + d * dy[k]);
    }
  }
  if (J)
    for (int r = 0; r < 2; ++r)
      for (int k = 0; k < 3; ++k)
        J[r][k] = du_dpc[r][0] * c.R[k] + du_dpc[r][1] * c.R[3 + k] + du_dpc[r][2] * c.R[6 + k];
}

struct UtState {
  float w4[4], R[3][3], s[3], M[3][3];
  float u[6], v[6], J[6][2][3];
  float mu, mv, dx[6], dy[6];
  float a0, b, c0;
};

__device__ void ut_forward_one(const UtArgs& A, int64_t i, UtState& S, bool jac) {
  const float* m = A.means + 3 * i;
  quat_rot(A.quats + 4 * i, S.w4, S.R);
  for (int k = 0; k < 3; ++k) S.s[k] = A.scales[3 * i + k];
  for (int r = 0; r < 3; ++r)
    for (int k = 0; k < 3; ++k) S.M[r][k] = gs_mul(S.R[r][k], S.s[k]);
  const float sq3 = gs_sqrt(3.0f);
  for (int j = 0; j < 6; ++j) {
    const int k = j % 3;
    const float sg = j < 3 ? 1.f : -1.f;
    const float p0 = gs_add(m[0], gs_mul(sq3, sg * S.M[0][k]));
    const float p1 = gs_add(m[1], gs_mul(sq3, sg * S.M[1][k]));
    const float p2 = gs_add(m[2], gs_mul(sq3, sg * S.M[2][k]));
    project_point(A.cam, A.lens, p0, p1, p2, S.u[j], S.v[j], jac ? S.J[j] : nullptr);
  }
  const float sixth = 1.0f / 6.0f;
  float su = S.u[0], sv = S.v[0];
  for (int j = 1; j < 6; ++j) { su = gs_add(su, S.u[j]); sv = gs_add(sv, S.v[j]); }
  S.mu = gs_mul(su, sixth);
  S.mv = gs_mul(sv, sixth);
  float sa = 0.f, sb = 0.f, sc = 0.f;
  for (int j = 0; j < 6; ++j) {
    S.dx[j] = gs_sub(S.u[j], S.mu);
    S.dy[j] = gs_sub(S.v[j], S.mv);
    sa = j ? gs_add(sa, gs_mul(S.dx[j], S.dx[j])) : gs_mul(S.dx[j], S.dx[j]);
    sb = j ? gs_add(sb, gs_mul(S.dx[j], S.dy[j])) : gs_mul(S.dx[j], S.dy[j]);
    sc = j ? gs_add(sc, gs_mul(S.dy[j], S.dy[j])) : gs_mul(S.dy[j], S.dy[j]);
  }
  S.a0 = gs_mul(sa, sixth);
  S.b = gs_mul(sb, sixth);
  S.c0 = gs_mul(sc, sixth);
}

__global__ void k_ut_fwd(const UtArgs A) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= A.n) return;
  UtState S;
  ut_forward_one(A, i, S, false);
  const float ca = gs_add(S.a0, A.blur), cc = gs_add(S.c0, A.blur);
  const float det = gs_sub(gs_mul(ca, cc), gs_mul(S.b, S.b));
  const float ds = gs_maxf(det, 1e-12f);
  A.conics[3 * i] = gs_div(cc, ds);
  A.conics[3 * i + 1] = gs_div(-S.b, ds);
  A.conics[3 * i + 2] = gs_div(ca, ds);
  float comp = 1.0f;
  if (A.aa) comp = gs_sqrt(gs_div(gs_maxf(gs_sub(gs_mul(S.a0, S.c0), gs_mul(S.b, S.b)), 0.0f), ds));
  const float mid = gs_mul(0.5f, gs_add(ca, cc));
  const float lam1 = gs_add(mid, gs_sqrt(gs_maxf(gs_sub(gs_mul(mid, mid), det), 0.01f)));
  const float radius = ceilf(gs_mul(3.0f, gs_sqrt(gs_maxf(lam1, 0.0f))));
  const float* m = A.means + 3 * i;
  const float z = cam_row(A.cam, 2, m[0], m[1], m[2]);
  const bool valid = (z > A.cam.znear) && (det > 0.0f);
  A.means2d[2 * i] = S.mu;
  A.means2d[2 * i + 1] = S.mv;
  A.depths[i] = z;
  A.radii[i] = valid ? radius : 0.0f;
  A.comp[i] = valid ? comp : 0.0f;
}

__global__ void k_ut_bwd(const UtArgs A) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= A.n) return;
  UtState S;
  ut_forward_one(A, i, S, true);
  const float gu = A.g_means2d ? A.g_means2d[2 * i] : 0.f, gv = A.g_means2d ? A.g_means2d[2 * i + 1] : 0.f;
  const float gA = A.g_conics ? A.g_conics[3 * i] : 0.f, gB = A.g_conics ? A.g_conics[3 * i + 1] : 0.f;
  const float gC = A.g_conics ? A.g_conics[3 * i + 2] : 0.f;
  const float gz = A.g_depths ? A.g_depths[i] : 0.f, gcomp = A.g_comp ? A.g_comp[i] : 0.f;
  const float* m = A.means + 3 * i;
  const float z = cam_row(A.cam, 2, m[0], m[1], m[2]);
  // conic / compensation -> (a0, b, c0), as the EWA projection's VJP
  const float a0 = S.a0, bb = S.b, c0 = S.c0;
  const float ca = a0 + A.blur, cc = c0 + A.blur;
  const float det = ca * cc - bb * bb;
  const float ds = fmaxf(det, 1e-12f), ids = 1.0f / ds;
  const bool valid = (z > A.cam.znear) && (det > 0.0f);
  float g_ca = gC * ids, g_cc = gA * ids, g_b = -gB * ids;
  float g_ds = -(gA * cc - gB * bb + gC * ca) * ids * ids;
  float g_a0 = 0.f, g_c0 = 0.f;
  if (A.aa && valid && gcomp != 0.0f) {
    const float det0r = a0 * c0 - bb * bb, det0 = fmaxf(det0r, 0.f), qv = det0 * ids, cm = sqrtf(qv);
    const float g_q = cm > 0.f ? gcomp * 0.5f / cm : 0.f;
    g_ds -= g_q * qv * ids;
    if (det0r > 0.f) {
      const float g_det0 = g_q * ids;
      g_a0 += g_det0 * c0;
      g_c0 += g_det0 * a0;
      g_b -= 2.f * bb * g_det0;
    }
  }
  const float g_det = det > 1e-12f ? g_ds : 0.f;
  g_ca += g_det * cc;
  g_cc += g_det * ca;
  g_b -= 2.f * bb * g_det;
  g_a0 += g_ca;
  g_c0 += g_cc;
  // sample moments -> sigma points (the mean's effect on sum dx_j vanishes)
  float gm[3] = {0.f, 0.f, 0.f}, gM[3][3] = {{0.f}};
  const float sq3 = sqrtf(3.0f);
  for (int j = 0; j < 6; ++j) {
    const float gu_j = (2.f * S.dx[j] * g_a0 + S.dy[j] * g_b + gu) / 6.f;
    const float gv_j = (2.f * S.dy[j] * g_c0 + S.dx[j] * g_b + gv) / 6.f;
    const int k = j % 3;
    const float sg = j < 3 ? 1.f : -1.f;
    for (int c = 0; c < 3; ++c) {
      const float gp = gu_j * S.J[j][0][c] + gv_j * S.J[j][1][c];
      gm[c] += gp;
      gM[c][k] += sg * sq3 * gp;
    }
  }
  gm[0] += gz * A.cam.R[6];
  gm[1] += gz * A.cam.R[7];
  gm[2] += gz * A.cam.R[8];
  float gR[3][3], gsc[3] = {0.f, 0.f, 0.f};
  for (int r = 0; r < 3; ++r)
    for (int k = 0; k < 3; ++k) {
      gR[r][k] = gM[r][k] * S.s[k];
      gsc[k] += gM[r][k] * S.R[r][k];
    }
  const float w = S.w4[0], a = S.w4[1], b = S.w4[2], c = S.w4[3];
  const float gw = 2.f * (-c * gR[0][1] + b * gR[0][2] + c * gR[1][0] - a * gR[1][2] - b * gR[2][0] + a * gR[2][1]);
  const float ga = 2.f * (b * gR[0][1] + c * gR[0][2] + b * gR[1][0] - 2.f * a * gR[1][1] - w * gR[1][2] +
                          c * gR[2][0] + w * gR[2][1] - 2.f * a * gR[2][2]);
  const float gb = 2.f * (-2.f * b * gR[0][0] + a * gR[0][1] + w * gR[0][2] + a * gR[1][0] + c * gR[1][2] -
                          w * gR[2][0] + c * gR[2][1] - 2.f * b * gR[2][2]);
  const float gc = 2.f * (-2.f * c * gR[0][0] - w * gR[0][1] + a * gR[0][2] + w * gR[1][0] - 2.f * c * gR[1][1] +
                          b * gR[1][2] + a * gR[2][0] + b * gR[2][1]);
  const float* q = A.quats + 4 * i;
  const float iqn = 1.0f / sqrtf(q[0] * q[0] + q[1] * q[1] + q[2] * q[2] + q[3] * q[3]);
  const float dot = w * gw + a * ga + b * gb + c * gc;
  A.g_quats[4 * i] = (gw - w * dot) * iqn;
  A.g_quats[4 * i + 1] = (ga - a * dot) * iqn;
  A.g_quats[4 * i + 2] = (gb - b * dot) * iqn;
  A.g_quats[4 * i + 3] = (gc - c * dot) * iqn;
  for (int k = 0; k < 3; ++k) {
    A.g_means[3 * i + k] = gm[k];
    A.g_scales[3 * i + k] = gsc[k];
  }
}

static int check_ut(const gs_camera* cam, const gs_lens* lens) {
  if (!cam || !lens) return set_error(GS_ERR_INVALID_ARG, "camera / lens is NULL");
  if (cam->width <= 0 || cam->height <= 0) return set_error(GS_ERR_INVALID_ARG, "camera size must be positive");
  if (lens->n_dist < 0 || lens->n_dist > 5) return set_error(GS_ERR_INVALID_ARG, "n_dist must be in [0, 5]");
  return GS_OK;
}

}  // namespace gs

using namespace gs;

extern "C" {

int gs_project_ut_forward(const gs_camera* cam, const gs_lens* lens, const float* means, const float* quats,
                          const float* scales, int64_t n, float blur, int antialias, float* means2d,
                          float* conics, float* depths, float* radii, float* compensation, void* stream) {
  clear_error();
  if (int e = check_ut(cam, lens)) return e;
  if (n <= 0) return GS_OK;
  if (!means || !quats || !scales || !means2d || !conics || !depths || !radii || !compensation)
    return set_error(GS_ERR_INVALID_ARG, "gs_project_ut_forward: NULL pointer");
  UtArgs A{};
  A.cam = *cam; A.lens = *lens; A.means = means; A.quats = quats; A.scales = scales; A.n = n;
  A.blur = blur; A.aa = antialias && blur > 0.0f;
  A.means2d = means2d; A.conics = conics; A.depths = depths; A.radii = radii; A.comp = compensation;
  k_ut_fwd<<<(unsigned)ceil_div(n, 128), 128, 0, as_stream(stream)>>>(A);
  return check_launch("k_ut_fwd");
}

int gs_project_ut_backward(const gs_camera* cam, const gs_lens* lens, const float* means, const float* quats,
                           const float* scales, int64_t n, float blur, int antialias, const float* g_means2d,
                           const float* g_conics, const float* g_depths, const float* g_compensation,
                           float* g_means, float* g_quats, float* g_scales, void* stream) {
  clear_error();
  if (int e = check_ut(cam, lens)) return e;
  if (n <= 0) return GS_OK;
  if (!means || !quats || !scales || !g_means || !g_quats || !g_scales)
    return set_error(GS_ERR_INVALID_ARG, "gs_project_ut_backward: NULL pointer");
  UtArgs A{};
  A.cam = *cam; A.lens = *lens; A.means = means; A.quats = quats; A.scales = scales; A.n = n;
  A.blur = blur; A.aa = antialias && blur > 0.0f;
  A.g_means2d = g_means2d; A.g_conics = g_conics; A.g_depths = g_depths; A.g_comp = g_compensation;
  A.g_means = g_means; A.g_quats = g_quats; A.g_scales = g_scales;
  k_ut_bwd<<<(unsigned)ceil_div(n, 128), 128, 0, as_stream(stream)>>>(A);
  return check_launch("k_ut_bwd");
}

}  // extern "C"
