// Load-time repack kernel (included inside namespace l3g, after
// l3g_matvec.cuh for Q8Tiles).
#pragma once

// ---------------------------------------------------------------------------
// Load-time repack: GGUF Q8_0 rows (34-byte blocks, already on the device)
// into the tiled layout.  Destination row r takes source row map(r):
// concatenation of up to three row ranges, or the interleave (a_i, b_i).
// Values are copied unchanged.
// ---------------------------------------------------------------------------
struct RepackArgs {
  const uint8_t* src[3];
  int src_row0[3];
  int seg_rows[3];
  int nseg;
  int interleave2;        // dst 2i <- seg0 row i, dst 2i+1 <- seg1 row i
  int src_blocks;         // blocks per source row
  int blk0;               // first source block of the column slice
  Q8Tiles dst;            // rows/cols of the destination
  uint8_t* out;
};

static __global__ void k_repack(const __grid_constant__ RepackArgs a) {
  const int nbc = a.dst.cols / 32;
  const long long total = (long long)a.dst.n_groups * a.dst.wr * nbc;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
       e += (long long)gridDim.x * blockDim.x) {
    const int r = (int)(e / nbc), b = (int)(e % nbc);
    const int g = r / a.dst.wr, i = r % a.dst.wr;
    const int bpt = a.dst.ck / 32;
    const int s = b / bpt, bb = b % bpt;
    uint8_t* tile = a.out + ((size_t)g * a.dst.nslices + s) * a.dst.tile_bytes;
    uint8_t* qd = tile + (size_t)i * a.dst.ck + bb * 32;
    uint8_t* dd = tile + (size_t)a.dst.wr * a.dst.ck + ((size_t)i * bpt + bb) * 2;
    const uint8_t* blk = nullptr;
    if (r < a.dst.rows) {
      int seg = 0, sr = r;
      if (a.interleave2) {
        seg = r & 1;
        sr = r >> 1;
      } else {
        while (seg < a.nseg - 1 && sr >= a.seg_rows[seg]) sr -= a.seg_rows[seg++];
      }
      blk = a.src[seg] + ((size_t)(a.src_row0[seg] + sr) * a.src_blocks + a.blk0 + b) * 34;
    }
    if (blk) {
      dd[0] = blk[0];
      dd[1] = blk[1];
#pragma unroll 8
      for (int j = 0; j < 32; ++j) qd[j] = blk[2 + j];
    } else {
      dd[0] = 0;
      dd[1] = 0;
      for (int j = 0; j < 32; ++j) qd[j] = 0;
    }
  }
}
