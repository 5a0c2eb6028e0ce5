// The reference's dtype promotion table (type_rules, matrix.h:166-180) as a constant, shared by the
// host-side mtxc_promote_types (shape.cpp) and the kernels that fuse a promotion into an op (mixed.cu),
// which use it at compile time to instantiate exactly the operand pairs the table allows.
#pragma once

namespace mtxc {

// in dtype-code order (F F16 U8 I32 I16 U32 U16 B I8 C64 BF16 I64 U64)
inline constexpr signed char kPromote[13][13] = {
    /* F    */ {0, 0, 0, 0, 0, 0, 0, 0, 0, 9, 0, 0, 0},
    /* F16  */ {0, 1, 0, 0, 0, 0, 0, 1, 0, 9, 0, 0, 0},
    /* U8   */ {0, 0, 2, 3, 4, 5, 6, 2, 4, 9, 0, 11, 12},
    /* I32  */ {0, 0, 3, 3, 3, 3, 3, 3, 3, 9, 0, 11, 0},
    /* I16  */ {0, 0, 4, 3, 4, 3, 3, 4, 4, 9, 0, 11, 0},
    /* U32  */ {0, 0, 5, 3, 3, 5, 5, 5, 3, 9, 0, 11, 12},
    /* U16  */ {0, 0, 6, 3, 3, 5, 6, 6, 3, 9, 0, 11, 12},
    /* B    */ {0, 1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12},
    /* I8   */ {0, 0, 4, 3, 4, 3, 3, 8, 8, 9, 0, 11, 0},
    /* C64  */ {9, 9, 9, 9, 9, 9, 9, 9, 9, 9, 9, 9, 9},
    /* BF16 */ {0, 0, 0, 0, 0, 0, 0, 10, 0, 9, 10, 0, 0},
    /* I64  */ {0, 0, 11, 11, 11, 11, 11, 11, 11, 9, 0, 11, 0},
    /* U64  */ {0, 0, 12, 0, 0, 12, 12, 12, 0, 9, 0, 0, 12},
};

constexpr int promote_code(int a, int b) {
    return (a < 0 || a > 12 || b < 0 || b > 12) ? -1 : kPromote[a][b];
}

}  // namespace mtxc
