#include "sx_tables.h"

namespace sx {

namespace {

// PAIR1 pair rows, n = 24..64: {mult, rot, mask0, mask1}.
const uint32_t kPair1[21][4] = {
    {0x58F41BF3u, 3, 0x8ED78C13u, 0x8EEE8C03u},  {0x58F41BF3u, 3, 0x8ED78C13u, 0x8EEE8C03u},
    {0x7AA2BE15u, 3, 0x8ED78C13u, 0x8ECE8C03u},  {0x7B229E11u, 3, 0x8ED78C13u, 0x8ECE8C03u},
    {0x3B22BE15u, 3, 0x8ED78C13u, 0x8ECE8C03u},  {0x46C63E17u, 19, 0x8F9A8E6Eu, 0x8E258FFEu},
    {0x46C63E17u, 19, 0x8F9A8E6Eu, 0x8E258FFEu}, {0x46C63E17u, 19, 0x8E6E8F9Au, 0x8E258FFEu},
    {0x46C63E17u, 19, 0x8F9A8E6Eu, 0x8E258FFEu}, {0xF75D60FFu, 19, 0x8E6E8F9Au, 0x8E258FFEu},
    {0xF75D60FFu, 19, 0x8E6E8F9Au, 0x8E258FFEu}, {0xF75D60FFu, 19, 0x8E6E8F9Au, 0x8E258FFEu},
    {0xF75D60FFu, 19, 0x8E6E8F9Au, 0x8E258FFEu}, {0xF75D60FFu, 19, 0x8E6E8F9Au, 0x8E258FFEu},
    {0xF75D60FFu, 19, 0x8E6E8F9Au, 0x8E258FFEu}, {0xF75D60FFu, 19, 0x8E6E8F9Au, 0x8E258FFEu},
    {0x82439F67u, 19, 0x8E6E8F9Au, 0x8E258FAEu}, {0xE2C7FC0Du, 19, 0x8F408FB0u, 0x8F918F89u},
    {0xE2C7FC0Du, 19, 0x8F408FA0u, 0x8F118FC9u}, {0xE2C7FC0Du, 19, 0x8F408FA0u, 0x8F118FC9u},
    {0xE2C7FC0Du, 19, 0x8F408FA0u, 0x8F118FC9u},
};

// spec1-w15, n = 16..128: {mult, mask}.
const uint32_t kSpec1W15[57][2] = {
    {0x84d1cf89u, 0x8fe08947u}, {0x84c1cf49u, 0x8fe48a47u}, {0x84d1cfe9u, 0x8fe08a47u}, {0x84d1cfc9u, 0x8ff08b67u},
    {0x84c1cf49u, 0x8fe08b47u}, {0x84c1cf99u, 0x8fa08b66u}, {0x862c1d37u, 0x8ff28c50u}, {0x84641fb7u, 0x8fa08c40u},
    {0x846c1fa7u, 0x8fe08c80u}, {0x844c1fd7u, 0x8ffe8c98u}, {0x846c1fa7u, 0x8ffe8d10u}, {0x845c1f77u, 0x8ffa8e10u},
    {0x843c1fa7u, 0x8ffe8e40u}, {0x843c1fa7u, 0x8ffe8e40u}, {0x842c1fc7u, 0x8fff8f00u}, {0x843c1fb7u, 0x8ffe8f10u},
    {0x84181fb5u, 0x8fe08f80u}, {0x84081f75u, 0x8ffa8f72u}, {0x84081f75u, 0x8fd68fd0u}, {0x84241f27u, 0x8ffc8fc0u},
    {0x84081f73u, 0x8fe08f80u}, {0x84081f75u, 0x8fbe8ff0u}, {0x3fed4cefu, 0x8fe08fe0u}, {0x3fed4cefu, 0x8fc18ff2u},
    {0x3fed4cefu, 0x8ff08ff0u}, {0x3fed4cefu, 0x8fe28ff0u}, {0x3fed4cefu, 0x8fe08fe0u}, {0x80081b7bu, 0x8ff08fc8u},
    {0x80081b7bu, 0x8ff48fc0u}, {0x400036cbu, 0x8f448fffu}, {0x400036cbu, 0x8fe48fffu}, {0x400036cbu, 0x8f448ff9u},
    {0x8000387bu, 0x8fe08ff7u}, {0x8000387bu, 0x8fc08feeu}, {0x80003779u, 0x8fe88ffeu}, {0x80003779u, 0x8fc88ffcu},
    {0x80003779u, 0x8fca8ffcu}, {0x80003779u, 0x8fcc8ffeu}, {0x80003879u, 0x8ffc8fefu}, {0x50003851u, 0x8ff98fffu},
    {0xd0003751u, 0x8ff98fffu}, {0x50003851u, 0x8ff98ff6u}, {0xd0003931u, 0x8ff98fffu}, {0xd0003931u, 0x8ff98ffau},
    {0xd0003931u, 0x8ff48ffau}, {0x300031b1u, 0x8ffb8ffcu}, {0x300031b1u, 0x8ffa8ffeu}, {0x300031b1u, 0x8ffb8ffcu},
    {0xc00031f1u, 0x8ffe8ffau}, {0x400031f1u, 0x8ffe8ffeu}, {0x400031f1u, 0x8ffe8ffeu}, {0x40003931u, 0x8ffc8ffcu},
    {0x40003931u, 0x8ffc8ffcu}, {0x40003931u, 0x8ff88ffeu}, {0x40003931u, 0x8ff88ffcu}, {0x80003811u, 0x8ffc8ffcu},
    {0x80003811u, 0x8ffc8ffcu},
};

// spec1-w16, n = 24..64.
const uint32_t kSpec1W16[21][2] = {
    {0x862d1c19u, 0x8fee8c30u}, {0x862d1d37u, 0x8fee8c30u}, {0x862d1d37u, 0x8ffe8c10u}, {0x842f1f37u, 0x8ffc8d10u},
    {0x840f1f67u, 0x8ffc8d10u}, {0x844f1f77u, 0x8ffe8d40u}, {0x840d1f37u, 0x8ffe8e10u}, {0x84091f33u, 0x8fe88e00u},
    {0x844d1f77u, 0x8fe08e00u}, {0x843c1fa7u, 0x8ffe8e40u}, {0x844c1f7fu, 0x8ffc8f02u}, {0x841c1fb9u, 0x8fe88f04u},
    {0x842c1fc7u, 0x8ffe8fd0u}, {0x83fc1fa3u, 0x8ffe8fd0u}, {0x83fc1fa3u, 0x8ffe8fc1u}, {0x83fc1fa3u, 0x8ffe8fd0u},
    {0x83fc1fa3u, 0x8fee8fc0u}, {0x84061f77u, 0x8fd08f80u}, {0x84081f6fu, 0x8ffe8fc0u}, {0x84081f25u, 0x8ffe8fe0u},
    {0x83f81f6fu, 0x8ff48fc0u},
};

}  // namespace

const TableDesc kTables[5] = {
    {"pair1-w16-v1", 3, 16, "c089b4eb", 4, 24, 21},
    {"spec1-w15", 2, 15, "37f72431", 2, 16, 57},
    {"spec1-w16", 2, 16, "753ffa03", 2, 24, 21},
    {"std1", 4, 15, "c5dba171", 2, 24, 21},
    {"spec1-test-per-rate", 2, 12, "a2f2fe40", 2, 16, 57},
};

bool table_row(int table, uint32_t n, uint32_t out[4]) {
    if (table < 0 || table > 4) return false;
    const TableDesc& t = kTables[table];
    if (n % 2 != 0 || n < t.n_lo) return false;
    const uint32_t i = (n - t.n_lo) / 2;
    if ((int)i >= t.rows) return false;
    out[0] = out[1] = out[2] = out[3] = 0;
    switch (table) {
        case 0:
            for (int k = 0; k < 4; k++) out[k] = kPair1[i][k];
            return true;
        case 1:
            out[0] = kSpec1W15[i][0];
            out[1] = kSpec1W15[i][1];
            return true;
        case 2:
            out[0] = kSpec1W16[i][0];
            out[1] = kSpec1W16[i][1];
            return true;
        case 3:  // std1: one pair at every rate
            out[0] = 0x840C1F37u;
            out[1] = 0x8FFE8FD0u;
            return true;
        case 4: {  // a different pair at every rate (the reference's syntheticPairs)
            static const uint32_t masks[4] = {0x8FFE8FD0u, 0x8FE08FC0u, 0x8FF08FE0u, 0x8F8E8FD8u};
            out[0] = 0x840C1F37u + (16u + 2u * i) * 0x2E0B5u;
            out[1] = masks[i % 4];
            return true;
        }
    }
    return false;
}

}  // namespace sx
