// Host-only harness for tests/test_tcx_plan_cpu.py: includes the short-M GEMV's
// translation unit and prints its plans (no GPU is touched). Each line:
// name m nw tile ks  tile_rows gx kb_per kblocks slice_rows issuers xi xa_stages tmem_cols smem part_bytes sc_off ok
//   xin wa raw_stages mma_stages
#include "../../gemma-4-webgpu-kernels_b200/csrc/gemv_tcx.cu"

#include <cstdio>

namespace {
struct Shape {
  const char *name;
  int n, k, bits, sg, nw;
};
}  // namespace

int main() {
  gq_ctx ctx;
  ctx.num_sms = 148;
  ctx.smem_optin = 232448;
  const Shape shapes[] = {{"qkv_l", 2560, 1536, 8, 1, 1}, {"q_g", 4096, 1536, 8, 1, 1},   {"o_l", 1536, 2048, 8, 1, 1},
                          {"o_g", 1536, 4096, 8, 1, 1},   {"gate_up", 6144, 1536, 4, 0, 2}, {"down", 1536, 6144, 2, 0, 1},
                          {"ple_gate", 256, 1536, 8, 1, 1}, {"ple_proj", 1536, 256, 8, 1, 1},
                          {"lm_head", 262144, 1536, 8, 1, 1}, {"odd", 300, 640, 8, 0, 1}, {"tiny", 77, 256, 4, 0, 1}};
  for (int m : {3, 5, 8, 16, 24, 33, 64})
    for (const Shape &sh : shapes) {
      gq_qweight w;
      w.n = sh.n;
      w.k = sh.k;
      w.bits = sh.bits;
      w.signed_i8 = sh.sg;
      w.group_size = sh.k;
      w.row_bytes = sh.bits == 8 ? sh.k : sh.k * sh.bits / 8;
      // tile 0 = default; ks 0 = the library's own choice (tcx_plan)
      for (int wa : {0, 1})
      for (int tile : {0, 16, 32, 64, 128})
        for (int ks : {0, 1, 2, 3, 4, 6, 8}) {
          if ((ks == 0 || wa) && tile != 0) continue;
          TcxPlan p{};
          const bool ok = ks == 0 ? tcx_plan(&ctx, &w, m, sh.nw, wa != 0, p)
                                  : tcx_plan_with(&ctx, &w, m, sh.nw, wa != 0, tile, ks, p);
          size_t sc_off = 0, part = 0;
          if (ok) {
            const TcxSmem L = tcx_layout(p.xa_stages, p.xa_tile, p.raw_stages, p.raw_bytes, p.mma_stages, p.mma_bytes,
                                         sh.nw * p.tile_rows * 4);
            sc_off = L.sc_off;
            part = (size_t)sh.nw * (size_t)m * (size_t)p.tile_rows * 8;
          }
          printf("%s %d %d %d %d  %d %d %d %d %d %d %d %d %d %zu %zu %zu %d  %d %d %d %d\n", sh.name, m, sh.nw, tile, ks,
                 p.tile_rows, p.gx, p.kb_per, p.kblocks, p.slice_rows, p.issuers, p.xi, p.xa_stages, p.tmem_cols,
                 p.smem, part, sc_off, ok ? 1 : 0, ok ? p.xin : 0, wa, p.raw_stages, p.mma_stages);
        }
    }
  return 0;
}
