// d3s_codes.cu - the audio codes output of a take (host code): the codebook
// columns of the sampled frame rows written as a 2-D .npy file, the format of
// npy_write_codes (src/npy.c:98-129) and of generate's Codes
// (src/generate.c:162-168): shape (n_codebooks, frames), codes[k][t] = column
// 1 + k of frame row t (column 0 is the main token), little-endian int64,
// C order, NumPy format 1.0 with the header padded to a multiple of 64 bytes.
#include <cstdio>
#include <cstring>

#include "d3s.h"
#include "d3s_kernels.cuh"

extern "C" int d3s_codes_write_npy(const char *path, const int32_t *frames, int n_frames,
                                   int width, int n_codebooks) {
  if (!path || n_frames < 0 || n_codebooks < 1 || width < 1 + n_codebooks ||
      (n_frames > 0 && !frames))
    return d3s::set_error(D3S_ERR_ARG, "codes: bad path / frames / width / n_codebooks");
  FILE *f = std::fopen(path, "wb");
  if (!f) return d3s::set_error(D3S_ERR_ARG, "codes: cannot open the output file");
  char header[128];
  const int n = std::snprintf(header, sizeof header,
                              "{'descr': '<i8', 'fortran_order': False, 'shape': (%d, %d), }",
                              n_codebooks, n_frames);
  const int pad = (64 - (10 + n + 1) % 64) % 64;  // magic + version + length, header, '\n'
  const int hlen = n + pad + 1;
  const unsigned char pre[10] = {0x93, 'N', 'U', 'M', 'P', 'Y', 1, 0,
                                 (unsigned char)(hlen & 0xFF), (unsigned char)(hlen >> 8)};
  bool ok = std::fwrite(pre, 1, 10, f) == 10 && std::fwrite(header, 1, (size_t)n, f) == (size_t)n;
  for (int i = 0; ok && i < pad; ++i) ok = std::fputc(' ', f) != EOF;
  ok = ok && std::fputc('\n', f) != EOF;
  for (int k = 0; ok && k < n_codebooks; ++k)
    for (int t = 0; ok && t < n_frames; ++t) {
      const long long v = frames[(size_t)t * width + 1 + k];
      unsigned char b[8];
      for (int i = 0; i < 8; ++i) b[i] = (unsigned char)((unsigned long long)v >> (8 * i));
      ok = std::fwrite(b, 1, 8, f) == 8;
    }
  ok = (std::fclose(f) == 0) && ok;
  if (!ok) return d3s::set_error(D3S_ERR_ARG, "codes: short write");
  return D3S_OK;
}
