// hxrun — block-chain runner with megarun's process protocol (hexagon/mega/megarun.cpp:1-4,132-195),
// on top of the libhxdit C ABI only.
//
//   hxrun HMXDIR [FIRST COUNT]
// loads HMXDIR/blkNN.bin for NN = FIRST .. FIRST+COUNT-1 (Anima fp16 or q8 packs, recognised by size),
// prints "ready", then serves stdin lines:
//   run X_IN EMB LORA CTX X_OUT [GH GW [SKIPMASK]]   ->  "done <ms>" | "error"
//   quit
// X_IN / X_OUT fp32 [D][T] (T = GH*GW, default 48x32), or the reference's 32x32-tile x32 layout when the
// name ends in ".x32"; EMB fp32 [2048]; LORA fp32 [6144]; CTX fp32 [1024][512]. Block k of the range is
// skipped when bit (FIRST + k) of SKIPMASK is set.
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <iostream>
#include <sstream>
#include <string>
#include <vector>

#include "../../include/hxdit.h"

namespace {

constexpr int D = 2048, NCTX = 512, CD = 1024, F = 8192, TMAX = 6144;

bool read_file(const std::string& p, std::vector<char>& out) {
  FILE* f = fopen(p.c_str(), "rb");
  if (!f) return false;
  fseek(f, 0, SEEK_END);
  const long n = ftell(f);
  fseek(f, 0, SEEK_SET);
  out.resize(n > 0 ? static_cast<size_t>(n) : 0);
  const bool ok = n >= 0 && fread(out.data(), 1, out.size(), f) == out.size();
  fclose(f);
  return ok;
}

bool write_file(const std::string& p, const void* data, size_t bytes) {
  FILE* f = fopen(p.c_str(), "wb");
  if (!f) return false;
  const bool ok = fwrite(data, 1, bytes, f) == bytes;
  return fclose(f) == 0 && ok;
}

bool ends_with(const std::string& s, const char* suf) {
  const size_t n = strlen(suf);
  return s.size() >= n && s.compare(s.size() - n, n, suf) == 0;
}

// [D][T] channel-major file <-> [T][D] rows; x32: tiles [T/32][D/32][32 rows][32 cols] (megarun.cpp:60-76)
void to_rows(const float* src, float* rows, int T, bool x32) {
  for (int t = 0; t < T; ++t)
    for (int c = 0; c < D; ++c)
      rows[static_cast<size_t>(t) * D + c] =
          x32 ? src[((static_cast<size_t>(t / 32) * (D / 32) + c / 32) * 1024) + (t % 32) * 32 + c % 32]
              : src[static_cast<size_t>(c) * T + t];
}
void from_rows(const float* rows, float* dst, int T, bool x32) {
  for (int t = 0; t < T; ++t)
    for (int c = 0; c < D; ++c) {
      const float v = rows[static_cast<size_t>(t) * D + c];
      if (x32)
        dst[((static_cast<size_t>(t / 32) * (D / 32) + c / 32) * 1024) + (t % 32) * 32 + c % 32] = v;
      else
        dst[static_cast<size_t>(c) * T + t] = v;
    }
}

uint16_t f2h(float f) {  // round-to-nearest-even fp32 -> fp16
  uint32_t x;
  std::memcpy(&x, &f, 4);
  const uint32_t sign = (x >> 16) & 0x8000u;
  x &= 0x7FFFFFFFu;
  if (x >= 0x7F800000u) return static_cast<uint16_t>(sign | (x > 0x7F800000u ? 0x7E00u : 0x7C00u));
  if (x >= 0x477FF000u) return static_cast<uint16_t>(sign | 0x7C00u);  // overflow to inf
  if (x < 0x38800000u) {                                               // subnormal or zero
    if (x < 0x33000000u) return static_cast<uint16_t>(sign);
    const uint32_t m = (x & 0x007FFFFFu) | 0x00800000u;
    const int shift = 113 - static_cast<int>(x >> 23);
    uint32_t h = m >> (shift + 13);
    const uint32_t rem = m & ((1u << (shift + 13)) - 1), half = 1u << (shift + 12);
    if (rem > half || (rem == half && (h & 1))) ++h;
    return static_cast<uint16_t>(sign | h);
  }
  uint32_t h = ((x - 0x38000000u) >> 13);
  const uint32_t rem = x & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1))) ++h;
  return static_cast<uint16_t>(sign | h);
}

}  // namespace

int main(int argc, char** argv) {
  if (argc < 2) {
    fprintf(stderr, "usage: hxrun HMXDIR [FIRST COUNT]\n");
    return 1;
  }
  const std::string dir = argv[1];
  const int first = argc > 2 ? atoi(argv[2]) : 0, count = argc > 3 ? atoi(argv[3]) : 28;
  if (count <= 0 || count > 64) {
    fprintf(stderr, "hxrun: bad block count\n");
    return 1;
  }
  hx_handle h = nullptr;
  if (hx_open(0, &h) != HX_OK) {
    fprintf(stderr, "hxrun: hx_open failed\n");
    return 1;
  }
  std::vector<int> wfds(count);
  const auto t0 = std::chrono::steady_clock::now();
  for (int i = 0; i < count; ++i) {
    char p[1024];
    snprintf(p, sizeof p, "%s/blk%02d.bin", dir.c_str(), first + i);
    std::vector<char> pack;
    if (!read_file(p, pack) || hx_weights_load(h, HX_MODEL_ANIMA, pack.data(), pack.size(), &wfds[i]) != HX_OK) {
      fprintf(stderr, "cannot load %s\n", p);
      hx_close(h);
      return 1;
    }
  }
  fprintf(stderr, "hxrun: weights loaded %.1fs\n",
          std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count());
  printf("ready\n");
  fflush(stdout);

  int blob = -1, blobT = 0, vecs = -1;
  int32_t meta[HX_A_NMETA_EXT];
  std::vector<float> rows, cs, sn;
  std::vector<uint16_t> ctx16(static_cast<size_t>(NCTX) * CD);
  if (hx_buf_alloc(h, (D + 3 * D) * sizeof(float), &vecs) != HX_OK) return 1;  // emb | lora
  void* vecs_dev = nullptr;
  hx_buf_ptr(h, vecs, &vecs_dev);
  std::string line;
  while (std::getline(std::cin, line)) {
    std::istringstream ss(line);
    std::string cmd;
    ss >> cmd;
    if (cmd == "quit") break;
    if (cmd != "run") continue;
    std::string xi, em, lo, cx, xo;
    int gh = 48, gw = 32;
    unsigned skipmask = 0;
    ss >> xi >> em >> lo >> cx >> xo;
    if (!(ss >> gh)) gh = 48;
    if (!(ss >> gw)) gw = 32;
    if (!(ss >> skipmask)) skipmask = 0;
    const int T = gh * gw;
    const auto ts = std::chrono::steady_clock::now();
    std::vector<char> xb, eb, lb, cb;
    const bool io = read_file(xi, xb) && read_file(em, eb) && read_file(lo, lb) && read_file(cx, cb);
    if (!io || T <= 0 || T % 32 || T > TMAX || xb.size() != static_cast<size_t>(D) * T * 4 || eb.size() != D * 4u ||
        lb.size() != 3u * D * 4 || cb.size() != static_cast<size_t>(CD) * NCTX * 4) {
      fprintf(stderr, "bad input T=%d\n", T);
      printf("error\n");
      fflush(stdout);
      continue;
    }
    size_t total = 0;
    if (hx_blob_layout(HX_MODEL_ANIMA, T, NCTX, 1, D, F, CD, meta, HX_A_NMETA_EXT, &total) != HX_OK) {
      printf("error\n");
      fflush(stdout);
      continue;
    }
    if (T > blobT) {
      if (blob >= 0) hx_buf_free(h, blob);
      blob = -1;
      if (hx_buf_alloc(h, total, &blob) != HX_OK) {
        fprintf(stderr, "blob alloc failed\n");
        printf("error\n");
        fflush(stdout);
        blobT = 0;
        continue;
      }
      blobT = T;
    }
    rows.resize(static_cast<size_t>(T) * D);
    to_rows(reinterpret_cast<const float*>(xb.data()), rows.data(), T, ends_with(xi, ".x32"));
    const float* ct = reinterpret_cast<const float*>(cb.data());  // [1024 ch][512 tok]
    for (int i = 0; i < NCTX; ++i)
      for (int c = 0; c < CD; ++c) ctx16[static_cast<size_t>(i) * CD + c] = f2h(ct[static_cast<size_t>(c) * NCTX + i]);
    cs.assign(static_cast<size_t>(T) * 64, 0.f);
    sn.assign(static_cast<size_t>(T) * 64, 0.f);
    hx_rope_anima(gh, gw, 10000.0, T, cs.data(), sn.data());
    int32_t rc = 0;
    bool ok = hx_buf_write(h, blob, meta[HX_A_X], rows.data(), rows.size() * 4) == HX_OK &&
              hx_buf_write(h, blob, meta[HX_A_CTX], ctx16.data(), ctx16.size() * 2) == HX_OK &&
              hx_buf_write(h, blob, meta[HX_A_COS], cs.data(), cs.size() * 4) == HX_OK &&
              hx_buf_write(h, blob, meta[HX_A_SIN], sn.data(), sn.size() * 4) == HX_OK &&
              hx_buf_write(h, vecs, 0, eb.data(), D * 4) == HX_OK &&
              hx_buf_write(h, vecs, D * 4, lb.data(), 3 * D * 4) == HX_OK;
    const float* emb_dev = static_cast<const float*>(vecs_dev);
    ok = ok && hx_chain(h, meta, HX_A_NMETA_EXT, wfds.data(), count, blob, nullptr, emb_dev, emb_dev + D,
                        skipmask >> first, 1, &rc) == HX_OK && rc == HX_OK;
    ok = ok && hx_buf_read(h, blob, meta[HX_A_X], rows.data(), rows.size() * 4) == HX_OK;
    int st = 0;
    ok = ok && hx_status(h, &st) == HX_OK && st == 0;
    if (!ok) {
      fprintf(stderr, "chain failed rc=%d\n", rc);
      printf("error\n");
      fflush(stdout);
      continue;
    }
    std::vector<float> out(rows.size());
    from_rows(rows.data(), out.data(), T, ends_with(xo, ".x32"));
    if (!write_file(xo, out.data(), out.size() * 4)) {
      printf("error\n");
      fflush(stdout);
      continue;
    }
    const double ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - ts).count();
    printf("done %.0f\n", ms);
    fflush(stdout);
  }
  hx_close(h);
  return 0;
}
