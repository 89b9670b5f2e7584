"""Initial conditions: geodesy, IC sampling and GPU seeding of FDM state rows.

* WGS84 geodesy (``geodetic_to_ecef``, ``ecef_to_geodetic``, ``ned_to_geodetic``) restated
  from the published formulas that the reference reaches through ``pymap3d``
  (R/cuda_fdm/rl_env.py:57-85 and the ``pm.ned2geodetic`` call at :166-174; pymap3d>=3.1,<4
  per requirements.txt): NED -> ENU -> ECEF offset about the origin, then an iterated
  geodetic latitude (fixed-point on the prime-vertical radius, run to convergence).
* ``seed_states`` builds 101-double FDM rows on the GPU (f16_seed_ic), replacing the CPU
  ``build_seed_vector`` loop (cuda_fdm/ic.py:117-138, 0.69 ms per aircraft on a CPU core).
* ``baseline_ics`` draws the synthetic IC distribution the benchmark configs are quoted on.
"""
import math
import re
from pathlib import Path

import numpy as np
import torch

from . import _lib

ORIGIN_LAT_DEG = 37.240778      # official BaseLat/BaseLon (R/cuda_fdm/rl_env.py:33-35)
ORIGIN_LON_DEG = 131.869556
ORIGIN_ALT_M = 0.0
WGS84_A_M = 6378137.0
WGS84_E2 = 0.0066943799901411   # pymap3d wgs84
FT2M = 0.3048
M2FT = 1.0 / FT2M

IC_COLUMNS = ("lat_deg", "lon_deg", "alt_ft", "vt_fps", "phi_deg", "theta_deg", "psi_deg",
              "alpha_deg", "beta_deg", "fuel_lbs", "fuelflow_pph", "geocentric")


# ---------------------------------------------------------------- WGS84 geodesy
def geodetic_to_ecef(lat_deg, lon_deg, h_m):
    lat = np.radians(lat_deg)
    lon = np.radians(lon_deg)
    sl, cl = np.sin(lat), np.cos(lat)
    N = WGS84_A_M / np.sqrt(1.0 - WGS84_E2 * sl * sl)
    return ((N + h_m) * cl * np.cos(lon), (N + h_m) * cl * np.sin(lon), (N * (1.0 - WGS84_E2) + h_m) * sl)


def ecef_to_geodetic(x, y, z, iters=12):
    """Geodetic latitude/longitude (deg) and ellipsoidal height (m), iterated to convergence."""
    x, y, z = (np.asarray(v, dtype=np.float64) for v in (x, y, z))
    p = np.hypot(x, y)
    lon = np.arctan2(y, x)
    lat = np.arctan2(z, p * (1.0 - WGS84_E2))
    for _ in range(iters):
        s = np.sin(lat)
        N = WGS84_A_M / np.sqrt(1.0 - WGS84_E2 * s * s)
        lat = np.arctan2(z + WGS84_E2 * N * s, p)
    s, c = np.sin(lat), np.cos(lat)
    N = WGS84_A_M / np.sqrt(1.0 - WGS84_E2 * s * s)
    h = np.where(np.abs(c) > 1e-12, p / np.where(np.abs(c) > 1e-12, c, 1.0) - N,
                 np.abs(z) - N * (1.0 - WGS84_E2))
    return np.degrees(lat), np.degrees(lon), h


def ned_to_geodetic(n, e, d, lat0=ORIGIN_LAT_DEG, lon0=ORIGIN_LON_DEG, h0=ORIGIN_ALT_M):
    """Cartesian NED (m) about (lat0, lon0, h0) -> geodetic lat, lon (deg), height (m)."""
    n, e, d = (np.asarray(v, dtype=np.float64) for v in (n, e, d))
    up = -d
    la, lo = math.radians(lat0), math.radians(lon0)
    t = math.cos(la) * up - math.sin(la) * n
    w = math.sin(la) * up + math.cos(la) * n
    dx = math.cos(lo) * t - math.sin(lo) * e
    dy = math.sin(lo) * t + math.cos(lo) * e
    x0, y0, z0 = geodetic_to_ecef(lat0, lon0, h0)
    return ecef_to_geodetic(x0 + dx, y0 + dy, z0 + w)


def official_seed_latlon(n, e, d):
    """The reference's official N/E/D -> seed lat/lon (deg) and MSL alt (ft): the tangent-derived
    height is discarded and MSL = -D (R/cuda_fdm/rl_env.py:166-174)."""
    lat, lon, _ = ned_to_geodetic(n, e, d)
    return lat, lon, -np.asarray(d, dtype=np.float64) * M2FT


# ---------------------------------------------------------------- ISA (for Mach -> true airspeed)
def _atm_tables():
    text = (Path(__file__).resolve().parent / "csrc" / "f16_tables.h").read_text()
    vals = re.search(r"#define F16_TAB_VALUES \\\n(.*?)\n\n", text, re.S).group(1)
    data = np.array([float(v) for v in vals.replace("\\", " ").replace("\n", " ").split(",")])
    off = {m.group(1): int(m.group(2)) for m in re.finditer(r"#define F16T_(\w+) (\d+)", text)}
    consts = {m.group(1): float(m.group(2)) for m in re.finditer(r"#define F16C_(\w+) \(([^)]+)\)", text)}
    return data, off, consts


def isa_sound_speed_fps(alt_ft):
    """Speed of sound (ft/s) of the reference ISA at geometric altitude alt_ft (fdm.cuh:174-224)."""
    data, off, c = _atm_tables()
    alt = np.asarray(alt_ft, dtype=np.float64)
    R = c["EarthRadius"]
    gp = (alt * R) / (R + alt)
    x = data[off["ATM_ALT"]:off["ATM_ALT"] + 9]
    y = data[off["ATM_TMP"]:off["ATM_TMP"] + 9]
    T = np.interp(np.maximum(gp, 0.0), x, y) + np.minimum(gp, 0.0) * data[off["ATM_LAPSE"]]
    return np.sqrt(c["SHRatio"] * c["Reng"] * T)


# ---------------------------------------------------------------- IC rows
def ic_rows(ic_list):
    """List of IC dicts (cuda_fdm/ic.py:117-120 keyword names) -> (n,12) float64 rows."""
    rows = np.zeros((len(ic_list), _lib.IC_N))
    for i, ic in enumerate(ic_list):
        rows[i, 0] = ic["lat_deg"]
        rows[i, 1] = ic["lon_deg"]
        rows[i, 2] = ic["alt_ft"]
        rows[i, 3] = ic["vt_fps"]
        rows[i, 4] = ic.get("phi_deg", 0.0)
        rows[i, 5] = ic.get("theta_deg", 0.0)
        rows[i, 6] = ic.get("psi_deg", 0.0)
        rows[i, 7] = ic.get("alpha_deg", 0.0)
        rows[i, 8] = ic.get("beta_deg", 0.0)
        rows[i, 9] = ic.get("fuel_lbs", 6000.0)
        rows[i, 10] = ic.get("fuelflow_pph", 0.0)
        rows[i, 11] = 0.0 if ic.get("lat_type", "geodetic") == "geodetic" else 1.0
        if ic.get("gamma_deg", 0.0) != 0.0:
            raise ValueError("gamma_deg is ignored by the reference seed builder; pass 0")
    return rows


def seed_states(ic, fcs_dt, device="cuda", out=None, layout=_lib.LAYOUT_SOA):
    """(n,12) IC rows (numpy or tensor) -> seeded FDM state on the GPU.

    Returns a (101, n) SoA tensor (or writes ``out``: (101, n) SoA or (n,101) AoS float64)."""
    lib = _lib.load()
    ic_t = torch.as_tensor(np.asarray(ic, dtype=np.float64) if not torch.is_tensor(ic) else ic,
                           dtype=torch.float64).to(device).contiguous()
    n = ic_t.shape[0]
    if out is None:
        out = torch.empty(_lib.STATE_N, n, dtype=torch.float64, device=device)
        layout = _lib.LAYOUT_SOA
    ld = out.shape[1] if layout == _lib.LAYOUT_SOA else _lib.STATE_N
    _lib.check(lib.f16_seed_ic(_lib.ptr(ic_t), n, _lib.ptr(out), layout, ld, float(fcs_dt),
                               _lib.stream_of(out)), "f16_seed_ic")
    return out


# ---------------------------------------------------------------- benchmark IC distribution
def baseline_ics(nenv, seed, sep_m=10_000.0, alt_km=(6.0, 9.0), mach=(0.6, 0.9), hdg_off_deg=30.0,
                 fuel_lbs=6000.0):
    """Seeded synthetic ICs of the benchmark configs: altitude U(6,9) km, Mach U(0.6,0.9)
    converted with the ISA speed of sound at that altitude, head-on along North at 10 km
    separation centred on the official origin, each heading offset by U(-30,30) deg,
    phi = theta = alpha = beta = 0, fuel 6000 lb.  Returns (2*nenv, 12) rows, even = ownship."""
    rng = np.random.default_rng(seed)
    alt_m = rng.uniform(alt_km[0], alt_km[1], nenv) * 1000.0
    m = rng.uniform(mach[0], mach[1], nenv)
    off = rng.uniform(-hdg_off_deg, hdg_off_deg, (nenv, 2))
    alt_ft = alt_m * M2FT
    vt = m * isa_sound_speed_fps(alt_ft)
    half = 0.5 * sep_m
    rows = np.zeros((2 * nenv, _lib.IC_N))
    for k, (north, hdg) in enumerate(((half, 180.0), (-half, 0.0))):
        lat, lon, altf = official_seed_latlon(np.full(nenv, north), np.zeros(nenv), -alt_m)
        r = rows[k::2]
        r[:, 0] = lat
        r[:, 1] = lon
        r[:, 2] = altf
        r[:, 3] = vt
        r[:, 6] = np.mod(hdg + off[:, k], 360.0)
        r[:, 9] = fuel_lbs
    return rows


# ---------------------------------------------------------------- counter-based action bins
_MASK = (1 << 64) - 1


def splitmix64_np(x):
    x = (np.asarray(x, dtype=np.uint64) + np.uint64(0x9E3779B97F4A7C15))
    x = (x ^ (x >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
    x = (x ^ (x >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
    return x ^ (x >> np.uint64(31))


def hash_bins_np(seed, decision, nac, num_bins=21):
    """(nac,4) uint8 action bins = splitmix64(seed, aircraft, decision, channel) % num_bins."""
    with np.errstate(over="ignore"):
        a = np.arange(nac, dtype=np.uint64)[:, None]
        c = np.arange(4, dtype=np.uint64)[None, :]
        key = (np.uint64(seed) * np.uint64(0x100000001B3)) ^ (np.uint64(decision) << np.uint64(40)) \
            ^ (a << np.uint64(2)) ^ c
        return (splitmix64_np(key) % np.uint64(num_bins)).astype(np.uint8)


def action_grid(num_bins=21, device="cpu"):
    """Reference action grid (R/cuda_fdm/ppo_gpu.py:178-180): float32 linspace(-1, 1, n) on
    `device` (torch's CPU and CUDA linspace round some interior bins differently)."""
    return torch.linspace(-1.0, 1.0, int(num_bins), device=device)


def bins_to_commands(bins, num_bins=21):
    """Reference action_to_env (R/cuda_fdm/ppo_gpu.py:361-369) on uint8/int bins -> float32 (N,4);
    the grid is built on the bins' device, as the reference does for grid=None."""
    grid = action_grid(num_bins, bins.device)
    cont = grid[bins.long()]
    ctrl = cont.clone()
    ctrl[:, 3] = 0.5 * cont[:, 3] + 0.5
    return ctrl
