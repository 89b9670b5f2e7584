#!/usr/bin/env python3
"""Generate ``f16_tables.h``: the F-16 coefficient data of JSBSim v1.0.0 in one packed array.

The numbers are the F-16 aerodynamic, engine, FCS-schedule and ISA-atmosphere data that the
reference flattens into ``cuda_fdm/gen/f16_gen.cuh`` (constants :9-60, tables :63-155, engine
table macros :159-161, FCS macros :164-167, ``f16_aero`` term list :170-238).  They are data
(the JSBSim ``f16.xml`` model), so they must be identical; the *layout* is ours:

* every table lives in one contiguous ``double`` array so a CUDA block can stage all of it
  into shared memory with one coalesced copy;
* the 25 lookups that share the 12-point angle-of-attack grid store that grid once and only
  their ordinate rows (``F16T_*`` offsets), so one segment search serves all of them;
* grids that several 2-D tables share (elevator, two beta grids, engine altitude grid) are
  stored once.

The generator checks every sharing assumption against the source and fails loudly if one
does not hold.  Run it only where the reference tree is available; the output is committed.

Usage: python gen_tables.py [path/to/f16_gen.cuh] [out.h]
"""
import re
import sys
from pathlib import Path

# The reference checkout: $F16_REFERENCE, else a "reference" directory beside this repository.
import os  # noqa: E402
REF_ROOT = Path(os.environ.get("F16_REFERENCE") or Path(__file__).resolve().parents[3] / "reference")
SRC_DEFAULT = str(REF_ROOT / "cuda_fdm" / "gen" / "f16_gen.cuh")


def parse(path):
    text = Path(path).read_text(encoding="utf-8")
    arrays = {m.group(1): [float(x) for x in m.group(3).split(",")]
              for m in re.finditer(r"__constant__ double (\w+)\[(\d+)\] = \{([^}]*)\};", text)}
    scalars = {m.group(1): float(m.group(2))
               for m in re.finditer(r"__constant__ double (\w+) = ([-+0-9.eE]+);", text)}
    return arrays, scalars


# name in our layout -> (source x array, source y array) for 1-D tables on the alpha grid
ALPHA_1D = [
    ("CDDLEF", "T1y_2"), ("CDDSB", "T1y_3"), ("CDQ", "T1y_4"), ("CDQ_DLEF", "T1y_5"),
    ("CYP", "T1y_7"), ("CYR", "T1y_8"),
    ("CLDLEF", "T1y_10"), ("CLDSB", "T1y_11"), ("CLQ", "T1y_12"), ("CLQ_DSB", "T1y_13"),
    ("CLP", "T1y_16"), ("CLR", "T1y_17"),
    ("CMDSB", "T1y_24"), ("CMQ", "T1y_25"),
    ("CNP", "T1y_28"), ("CNR", "T1y_29"),
]
ALPHA_1D_X = ["T1x_2", "T1x_3", "T1x_4", "T1x_5", "T1x_7", "T1x_8", "T1x_10", "T1x_11",
              "T1x_12", "T1x_13", "T1x_16", "T1x_17", "T1x_24", "T1x_25", "T1x_28", "T1x_29"]
# 2-D tables with alpha rows: name -> (row array, col array, data array, column-grid group)
ALPHA_2D = [
    ("CDDH", "T2r_0", "T2c_0", "T2d_0", "ELEV"),
    ("CLDH", "T2r_9", "T2c_9", "T2d_9", "ELEV"),
    ("CMDH", "T2r_22", "T2c_22", "T2d_22", "ELEV"),
    ("CLB", "T2r_14", "T2c_14", "T2d_14", "BETA13"),
    ("CNB", "T2r_26", "T2c_26", "T2d_26", "BETA13"),
    ("CLDA", "T2r_18", "T2c_18", "T2d_18", "BETA7"),
    ("CLDR", "T2r_21", "T2c_21", "T2d_21", "BETA7"),
    ("CNDA", "T2r_31", "T2c_31", "T2d_31", "BETA7"),
    ("CNDR", "T2r_32", "T2c_32", "T2d_32", "BETA7"),
]
# 1-D tables on their own (Mach / schedule) grids: name -> (x array, y array)
OTHER_1D = [
    ("CDMACH", "T1x_1", "T1y_1"), ("CYB_M", "T1x_6", "T1y_6"), ("CLB_M", "T1x_15", "T1y_15"),
    ("CLDA_M", "T1x_19", "T1y_19"), ("CLDR_M", "T1x_20", "T1y_20"), ("CMA_M", "T1x_23", "T1y_23"),
    ("CNB_M", "T1x_27", "T1y_27"), ("CNDA_M", "T1x_30", "T1y_30"), ("CNDR_M", "T1x_33", "T1y_33"),
    ("FCS_AIL_SPEED", "T1x_37", "T1y_37"), ("FCS_ELEV_SCHED", "T1x_38", "T1y_38"),
    ("FCS_YAW_RATE", "T1x_39", "T1y_39"), ("KCLGE", "T1x_40", "T1y_40"),
]
# engine thrust tables (Mach rows x density-altitude columns)
ENGINE_2D = [("ENG_IDLE", "T2r_34", "T2c_34", "T2d_34"),
             ("ENG_MIL", "T2r_35", "T2c_35", "T2d_35"),
             ("ENG_AUG", "T2r_36", "T2c_36", "T2d_36")]
ATMOS = [("ATM_ALT", "ATM_ALT"), ("ATM_TMP", "ATM_TMP"), ("ATM_LAPSE", "ATM_LAPSE"),
         ("ATM_PBRK", "ATM_PBRK"), ("ATM_DBRK", "ATM_DBRK")]
# the nine Mach-indexed aerodynamic tables, also stored resampled on the union of their grids
MACH_1D = ["CDMACH", "CYB_M", "CLB_M", "CLDA_M", "CLDR_M", "CMA_M", "CNB_M", "CNDA_M", "CNDR_M"]


def table1d(x, y, k):
    """The reference's table1d (end clamps, linear inside) evaluated in double."""
    if k <= x[0]:
        return y[0]
    if k >= x[-1]:
        return y[-1]
    r = 1
    while r < len(x) - 1 and x[r] < k:
        r += 1
    f = min((k - x[r - 1]) / (x[r] - x[r - 1]), 1.0)
    return f * (y[r] - y[r - 1]) + y[r - 1]


def build(arrays, scalars):
    data = []
    offs = {}   # name -> (offset, length)

    def put(name, vals):
        offs[name] = (len(data), len(vals))
        data.extend(vals)

    alpha = arrays["T1x_2"]
    assert len(alpha) == 12
    for nm in ALPHA_1D_X:
        assert arrays[nm] == alpha, nm
    for _, r, _, _, _ in ALPHA_2D:
        assert arrays[r] == alpha, r
    put("ALPHA", alpha)
    for name, y in ALPHA_1D:
        assert len(arrays[y]) == 12
        put(name, arrays[y])
    groups = {}
    for name, _, c, d, grp in ALPHA_2D:
        if grp in groups:
            assert arrays[c] == arrays[groups[grp]], (name, grp)
        else:
            groups[grp] = c
            put("GRID_" + grp, arrays[c])
        assert len(arrays[d]) == 12 * len(arrays[c])
        put(name, arrays[d])
    for name, x, y in OTHER_1D:
        assert len(arrays[x]) == len(arrays[y])
        put(name + "_X", arrays[x])
        put(name + "_Y", arrays[y])
    eng_cols = arrays["T2c_34"]
    put("GRID_DENSALT", eng_cols)
    for name, r, c, d in ENGINE_2D:
        assert arrays[c] == eng_cols, name
        assert len(arrays[d]) == len(arrays[r]) * len(arrays[c])
        put(name + "_MACH", arrays[r])
        put(name, arrays[d])
    for name, src in ATMOS:
        put(name, arrays[src])
    # Resampled Mach tables: a piecewise-linear table evaluated at a superset of its breakpoints
    # and interpolated linearly again is the same function (end clamps included, since every
    # grid lies inside the union's range), so the nine lookups can share one segment search.
    srcs = {name: (x, y) for name, x, y in OTHER_1D}
    union = sorted({v for name in MACH_1D for v in arrays[srcs[name][0]]})
    put("MACHU", union)
    for name in MACH_1D:
        x, y = arrays[srcs[name][0]], arrays[srcs[name][1]]
        assert x == sorted(x) and x[0] >= union[0] and x[-1] <= union[-1], name
        put("MU_" + name, [table1d(x, y, u) for u in union])
    used = set(ALPHA_1D_X) | {y for _, y in ALPHA_1D} | {"T1x_2"}
    for _, r, c, d, _ in ALPHA_2D:
        used |= {r, c, d}
    for _, x, y in OTHER_1D:
        used |= {x, y}
    for _, r, c, d in ENGINE_2D:
        used |= {r, c, d}
    used |= {s for _, s in ATMOS}
    missing = set(arrays) - used
    assert not missing, f"unplaced source arrays: {sorted(missing)}"
    return data, offs


def emit(data, offs, scalars, src):
    lines = [
        "// GENERATED by gen_tables.py -- do not edit.",
        "// F-16 coefficient, engine, FCS-schedule and ISA data of JSBSim v1.0.0 (f16.xml), packed",
        "// into one array (F16_TAB) for one-copy shared-memory staging. Offsets: F16T_<name>,",
        "// lengths: F16N_<name>. Alpha-grid tables store only their ordinates (grid = F16T_ALPHA).",
        f"// Source of the numbers: the reference's {Path(src).name}.",
        "#ifndef F16_TABLES_H",
        "#define F16_TABLES_H",
        "",
        f"#define F16_TAB_LEN {len(data)}",
    ]
    for name, (o, n) in offs.items():
        lines.append(f"#define F16T_{name} {o}")
        lines.append(f"#define F16N_{name} {n}")
    lines.append("")
    lines.append("// physical / engine constants (reference f16_gen.cuh:9-60)")
    for name, v in scalars.items():
        lines.append(f"#define F16C_{name} ({v!r})")
    lines.append("")
    lines.append("#define F16_TAB_VALUES \\")
    row = []
    for i, v in enumerate(data):
        row.append(repr(v))
        if len(row) == 8 or i == len(data) - 1:
            tail = "," if i != len(data) - 1 else ""
            lines.append("  " + ", ".join(row) + tail + (" \\" if i != len(data) - 1 else ""))
            row = []
    lines.append("")
    lines.append("#endif  // F16_TABLES_H")
    return "\n".join(lines) + "\n"


def main():
    src = sys.argv[1] if len(sys.argv) > 1 else SRC_DEFAULT
    out = Path(sys.argv[2]) if len(sys.argv) > 2 else Path(__file__).with_name("f16_tables.h")
    arrays, scalars = parse(src)
    data, offs = build(arrays, scalars)
    out.write_text(emit(data, offs, scalars, src), encoding="utf-8")
    print(f"wrote {out} ({len(data)} doubles, {len(offs)} tables, {len(scalars)} constants)")


if __name__ == "__main__":
    main()
