// panel.h — the row-stationary execution layout ("vector panels").
//
// The reference's VCSR (include/vcsr.hpp) is segment-major: a group holds one
// column segment of `bundle` rows, so every (row, segment) pair costs one
// read-modify-write of a C row (src/kernels.cu:92-98).  The B200 layout
// keeps C stationary instead: rows are taken `R` at a time ("a vector"), and
// the vector sweeps the union of its rows' columns in ascending order.  Per
// union column j it stores the column index ucol[j] and the R values
// uval[j*R .. j*R+R) (zero where a row lacks the column), so one 16..64-byte
// load feeds R rows and one B row load feeds R*4 FMAs per lane.  R = 1 is
// plain CSR order.  Equal columns inside one row (duplicates) stay separate
// union entries (keyed by (column, occurrence)), so every row sums its
// entries in CSR order.
//
// Work is cut into nnz-balanced units of at most `chunk` union columns.  A
// vector longer than that is split over several units ("split vector"); each
// part writes its R x O partial sums to scratch and the last part to finish
// adds the parts in fixed order and writes C (deterministic, no waiting).
#pragma once
#include <cstdint>
#include <vector>

#include "vcsr_spmm.h"

namespace vcsr {

struct Unit {    // one work unit = (vector, union range, split slot)
  int vec;       // vector id (rows vec*R .. vec*R+R-1)
  int begin;     // first union index
  int end;       // one past the last union index
  int slot;      // -1 when the vector is not split, else its part's slot
};

struct SplitPart {  // per split slot
  int sv;           // split-vector id
  int part;         // part index within the vector
};

struct SplitVec {   // per split vector
  int first_slot;   // slot of part 0 (parts are consecutive slots)
  int nparts;
};

struct PanelHost {
  int R = 1;
  int num_vectors = 0;
  int chunk = 0;
  std::vector<int> vec_ptr;  // num_vectors + 1 offsets into ucol
  std::vector<int> ucol;     // union column per entry
  std::vector<float> uval;   // R values per entry
  std::vector<uint32_t> umask;  // R > 1: bit r = row r holds the entry (else padding)
  std::vector<Unit> units;
  std::vector<SplitPart> parts;
  std::vector<SplitVec> svecs;
};

// Union sizes per candidate R on a sample of 16-row windows; returns the
// largest R <= 8 whose vectors are at least 60% dense.
int choose_vec_rows(const vcsr_csr &csr, double *density_out);

// Build the layout on the host for a given R (1, 2, 4, 8, 16).  chunk <= 0
// picks min(union columns / (sms * 32), max(512, 2 x average vector)) clamped
// to [256, 2048], so that a wave of sub-warps holds many units and rows much
// longer than the average (power-law hubs) are split over several warps.
vcsr_status build_panel_host(const vcsr_csr &csr, int R, int chunk, int sms,
                             PanelHost *out);

}  // namespace vcsr
