// The STQ codebook tables the library decodes with: one row of constants per even rate n.
// Data from the reference's pack contract (src/exl3/codebook_tables.zig:101-214 and the PAIR1
// rows of src/exl3/expert_exl3.zig:24-46); each table's rows are pinned by the reference's
// sha256 digests in the tests (tests/test_capi_host.py), so a changed constant fails there.
#pragma once

#include <stdint.h>

namespace sx {

struct TableDesc {
    const char* name;
    int codebook;      // sx_codebook
    int window_bits;   // window the rows were tuned at (PAIR1 decodes at this window only)
    const char* digest;
    int fields;        // constants per row the codebook reads
    uint32_t n_lo;     // rate of row 0; row i is n_lo + 2i
    int rows;
};

// The four shipped tables plus the reference's test-only per-rate SPEC1 table.
extern const TableDesc kTables[5];

// The row of `table` at rate n: {mult, mask} for STD1/SPEC1, {mult, rot, mask0, mask1} for PAIR1.
// Returns false where the table has no row.
bool table_row(int table, uint32_t n, uint32_t out[4]);

}  // namespace sx
