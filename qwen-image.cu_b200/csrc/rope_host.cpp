// rope_host.cpp -- the 3-axis RoPE table Qwen-Image feeds the transformer.
//
// Restates rope.h (gen_qwen_image_pe :175-180 -> gen_qwen_image_ids :159-172
// -> gen_flux_img_ids with scale_rope :119-156 -> embed_nd :89-116 -> rope
// :25-47) with the same single-precision expressions, so the table matches the
// reference's host computation.  Layout [n_txt + n_img][64 pairs][2][2] FP32,
// text positions first, each pair [cos, -sin, sin, cos]; axes {16, 56, 56},
// theta 10000.  h, w are latent sizes (2x2 patches).
#include <cmath>
#include <vector>

#include "../../include/qwen_image_b200.h"

namespace qi {

static std::vector<float> linspace_f(float start, float end, int num) {
  std::vector<float> r(num);
  if (num == 1) {
    r[0] = start;
    return r;
  }
  const float step = (end - start) / (num - 1);
  for (int i = 0; i < num; ++i) r[i] = start + i * step;
  return r;
}

int rope_table_host(int h, int w, int n_txt, float* pe) {
  const int patch = 2;
  const int axes[3] = {16, 56, 56};
  const float theta = 10000.0f;
  const int h_len = (h + patch / 2) / patch;
  const int w_len = (w + patch / 2) / patch;
  const int n = n_txt + h_len * w_len;
  std::vector<float> ids(static_cast<size_t>(n) * 3);
  const int txt_start = h_len > w_len ? h_len : w_len;
  if (n_txt > 0) {
    std::vector<float> tl = linspace_f(static_cast<float>(txt_start), static_cast<float>(n_txt + txt_start), n_txt);
    for (int j = 0; j < n_txt; ++j) ids[3 * j] = ids[3 * j + 1] = ids[3 * j + 2] = tl[j];
  }
  const int hs = -(h_len / 2), ws = -(w_len / 2);
  std::vector<float> rows = linspace_f(static_cast<float>(hs), static_cast<float>(hs + h_len - 1), h_len);
  std::vector<float> cols = linspace_f(static_cast<float>(ws), static_cast<float>(ws + w_len - 1), w_len);
  for (int i = 0; i < h_len; ++i)
    for (int j = 0; j < w_len; ++j) {
      const int p = n_txt + i * w_len + j;
      ids[3 * p] = 0.0f;
      ids[3 * p + 1] = rows[i];
      ids[3 * p + 2] = cols[j];
    }
  int off = 0;
  for (int a = 0; a < 3; ++a) {
    const int dim = axes[a], hd = dim / 2;
    std::vector<float> sc = linspace_f(0.0f, (dim * 1.0f - 2.0f) / dim, hd);
    std::vector<float> omega(hd);
    for (int j = 0; j < hd; ++j) omega[j] = 1.0f / std::pow(theta, sc[j]);
    for (int p = 0; p < n; ++p)
      for (int j = 0; j < hd; ++j) {
        const float ang = ids[3 * p + a] * omega[j];
        float* e = pe + static_cast<size_t>(p) * 256 + static_cast<size_t>(off + j) * 4;
        e[0] = std::cos(ang);
        e[1] = -std::sin(ang);
        e[2] = std::sin(ang);
        e[3] = std::cos(ang);
      }
    off += hd;
  }
  return QI_OK;
}

}  // namespace qi
