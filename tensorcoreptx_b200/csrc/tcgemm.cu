// tcgemm.cu -- host side of libtcgemm.so: the C ABI declared in include/tcgemm.h.
//
// Plays the role of the reference's solver*.cu + per-kernel launch_kernel
// (src/solver.cu:6-28, kernels/*.cu launch wrappers): validates the problem,
// picks the tile shape and schedule, encodes the TMA descriptors and launches
// the tcgen05 kernel on the caller's stream.  Unlike the reference it never
// exits the process: every failure is a tcg_status.
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdio>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "../../include/tcgemm.h"
#include "tcg_gemm_kernel.cuh"
#include "tcg_quant.cuh"

namespace {

using namespace tcg;

constexpr int kMaxDevices = 64;

thread_local int t_last_cuda_error = 0;
thread_local int t_last_tile_n = 0;
thread_local int t_last_tile_m = 0;
std::atomic<unsigned long long> g_timeout_ns{2000000000ull};
std::atomic<int> g_force_bn{0};
std::atomic<int> g_force_pair{0};

struct DeviceState {
    std::once_flag once;
    bool supported = false;
    int sms = 0;
    std::mutex mu;
    cudaMemPool_t pool = nullptr;  // private pool for the int4 workspace
};
DeviceState g_dev[kMaxDevices];

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*,
                                  CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                  CUtensorMapFloatOOBfill);
EncodeTiledFn g_encode = nullptr;
std::once_flag g_encode_once;

tcg_status cuda_fail(cudaError_t e)
{
    t_last_cuda_error = static_cast<int>(e);
    return TCG_ERR_CUDA;
}

tcg_status device_state(DeviceState** out)
{
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e);
    if (dev < 0 || dev >= kMaxDevices) return TCG_ERR_UNSUPPORTED;
    DeviceState& d = g_dev[dev];
    std::call_once(d.once, [&]() {
        int major = 0, minor = 0;
        cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
        cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
        d.supported = (major == 10 && minor == 0);
    });
    if (!d.supported) return TCG_ERR_UNSUPPORTED;
    *out = &d;
    return TCG_SUCCESS;
}

tcg_status resolve_encode()
{
    std::call_once(g_encode_once, []() {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_encode = reinterpret_cast<EncodeTiledFn>(fn);
    });
    return g_encode ? TCG_SUCCESS : TCG_ERR_CUDA;
}

// Recently encoded tensor maps, per host thread (no locking): a map depends
// only on its arguments, so calls that repeat a buffer and shape -- the
// common case for GEMMs in a loop -- skip the driver's encoder.
struct MapKey {
    const void* base;
    uint64_t d0, d1, d2, s1, s2;
    uint32_t box0, box1;
    int dt;
    int swz;
    bool operator==(const MapKey& o) const
    {
        return base == o.base && d0 == o.d0 && d1 == o.d1 && d2 == o.d2 && s1 == o.s1 && s2 == o.s2 &&
               box0 == o.box0 && box1 == o.box1 && dt == o.dt && swz == o.swz;
    }
};
struct MapCache {
    static constexpr int kEntries = 16;
    MapKey key[kEntries];
    CUtensorMap map[kEntries];
    bool used[kEntries] = {};
    int next = 0;
};
thread_local MapCache t_map_cache;

tcg_status encode_3d_uncached(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t d0, uint64_t d1,
                              uint64_t d2, uint64_t s1, uint64_t s2, uint32_t box0, uint32_t box1,
                              CUtensorMapSwizzle swz);

// 3-D tiled map: dims {d0 (contiguous), d1, d2}, byte strides of d1 and d2;
// 128-byte swizzle unless asked otherwise.
tcg_status encode_3d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t d0, uint64_t d1,
                     uint64_t d2, uint64_t s1, uint64_t s2, uint32_t box0, uint32_t box1,
                     CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B)
{
    const MapKey k{base, d0, d1, d2, s1, s2, box0, box1, static_cast<int>(dt), static_cast<int>(swz)};
    MapCache& c = t_map_cache;
    for (int i = 0; i < MapCache::kEntries; ++i) {
        if (c.used[i] && c.key[i] == k) {
            *map = c.map[i];
            return TCG_SUCCESS;
        }
    }
    const tcg_status s = encode_3d_uncached(map, dt, base, d0, d1, d2, s1, s2, box0, box1, swz);
    if (s == TCG_SUCCESS) {
        const int i = c.next;
        c.next = (c.next + 1) % MapCache::kEntries;
        c.key[i] = k;
        c.map[i] = *map;
        c.used[i] = true;
    }
    return s;
}

tcg_status encode_3d_uncached(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t d0, uint64_t d1,
                              uint64_t d2, uint64_t s1, uint64_t s2, uint32_t box0, uint32_t box1,
                              CUtensorMapSwizzle swz)
{
    cuuint64_t dims[3] = {d0, d1, d2};
    cuuint64_t strides[2] = {s1, s2};
    cuuint32_t box[3] = {box0, box1, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = g_encode(map, dt, 3, const_cast<void*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        t_last_cuda_error = static_cast<int>(r);
        return TCG_ERR_CUDA;
    }
    return TCG_SUCCESS;
}

// Tile shape.  Problems that fill a wave of SM pairs with 512 x 256 tiles
// use that pair-wide tile.  Below that the candidates are CTA-pair 256 x BN
// tiles (BN 256/128, one pair per two SMs) and single-CTA 128 x BN tiles
// (BN 256/128/64, one per SM), with
// cost = waves of resident units x BN / efficiency, the critical path in
// units of one SM's 128-column share of a tile, where efficiency is the
// measured per-SM throughput of the shape relative to the 256 x 256 pair
// (int8 on B200, 4096..16384 cubed: the pair reads a third less operand data
// per MAC than a single 128 x 256 tile, and 128-wide tiles issue half-width
// MMAs).  Ties go to the earlier (more efficient) shape.
struct TileChoice {
    int bn;
    int shape;  // kShapeSingle / kShapePair / kShapeWide
};

// Environment overrides (read once; the tcg_set_* calls take precedence):
// TCG_TILE_N = 64|128|256, TCG_CTA_PAIR = 1 (single) | 2 (pair),
// TCG_GROUP_M = band height in tiles, TCG_K_ALT = 0|1, TCG_UNITS = at most
// this many persistent CTAs (pairs of CTAs for pair tiles), TCG_TMA_STORE = 0
// (write C with plain stores instead of TMA stores), TCG_TAIL_SPLIT = 0 (no
// half tiles in the last wave), TCG_STATIC_SCHEDULE = 1 (persistent units
// with round-robin work items instead of cluster launch control), TCG_PDL = 0
// (no programmatic dependent launch), TCG_STREAM_K = 1 (stream-K split of
// partial waves for integer kinds), TCG_S4_PREPASS = 1 (int4 in two passes).
int env_int(const char* name, int dflt = 0)
{
    const char* v = std::getenv(name);
    return v ? std::atoi(v) : dflt;
}

bool pdl_enabled()
{
    static const int env_pdl = env_int("TCG_PDL", 1);
    return env_pdl != 0;
}

TileChoice choose_tile(int M, int N, int K, int elem_bytes, int batches, int sms, bool i8_mn)
{
    static const int env_bn = env_int("TCG_TILE_N");
    static const int env_pair = env_int("TCG_CTA_PAIR");
    const int forced_bn = g_force_bn.load() ? g_force_bn.load() : env_bn;
    // 0 auto, 1 single, 2 pair, 3 wide, 4 pair-wide
    const int forced = g_force_pair.load() ? g_force_pair.load() : env_pair;
    struct Cand {
        int shape;
        int bn;
        double eff;
    };
    static const Cand cands[] = {{kShapePair, 256, 1.00}, {kShapeSingle, 256, 0.87}, {kShapePair, 128, 0.72},
                                 {kShapeSingle, 128, 0.72}, {kShapeSingle, 64, 0.50}};
    // Measured on B200 (int8 and fp16, 4096..32768 cubed, work items handed
    // out in order by cluster launch control): the pair 512 x 256 tile --
    // the least operand traffic from L2 per MAC (48 bytes per clock per SM at
    // the int8 rate, against 64 for 256 x 256 tiles) -- is the fastest shape
    // once it fills a wave of SM pairs (int8 8192^3: 3202 TOPS against 3029
    // for pair 256 x 256 and 3071 for wide; fp16 8192^3: 1512 against 1393
    // and 1473 TFLOP/s); at int8 4096^3 its 1.73 waves cost what the traffic
    // saves (all shapes within 1 %).  Smaller problems are sized by waves.
    const long long pw_tiles = static_cast<long long>((M + 511) / 512) * ((N + 255) / 256) * batches;
    if (forced == 4 || (!forced && !forced_bn && pw_tiles >= sms / 2)) return TileChoice{256, kShapePairWide};
    if (forced == 3) return TileChoice{256, kShapeWide};
    TileChoice best{256, kShapePair};
    double best_cost = -1.0;
    for (const Cand& c : cands) {
        const bool pair = c.shape == kShapePair;
        if ((forced == 1 && pair) || (forced == 2 && !pair)) continue;
        if (forced_bn && c.bn != forced_bn) continue;
        if (i8_mn && (pair ? c.bn / 2 : c.bn) < 128) continue;  // whole 128-byte atoms
        const long long tm = (M + (pair ? 255 : 127)) / (pair ? 256 : 128);
        const long long tiles = tm * ((N + c.bn - 1) / c.bn) * batches;
        const long long units = pair ? sms / 2 : sms;
        const long long waves = (tiles + units - 1) / units;
        const double cost = static_cast<double>(waves) * c.bn / c.eff;
        if (best_cost < 0 || cost < best_cost) {
            best = TileChoice{c.bn, c.shape};
            best_cost = cost;
        }
    }
    if (best_cost < 0) best = TileChoice{forced_bn ? forced_bn : 256, forced == 1 ? kShapeSingle : kShapePair};
    return best;
}

// Band height: about square in elements, gm * tile_m ~ gn * BN with gm * gn =
// the units running at once, so a wave touches as few operand panels as it
// can (pair 256 x 256: 8; single 128 x 256: 16).
int choose_group_m(int tile_m, int bn, int units, int tiles_m)
{
    static const int env_g = env_int("TCG_GROUP_M");
    int g = env_g;
    if (g <= 0) {
        const double ideal = std::sqrt(static_cast<double>(units) * bn / tile_m);
        g = 1;
        while (g * 2 <= ideal) g *= 2;
    }
    if (g > tiles_m) g = tiles_m;
    return g < 1 ? 1 : g;
}

// Epilogue options: further destinations of C (peer buffers) and the
// dequantisation scales (device pointers).
struct EpiArgs {
    void* const* extra = nullptr;
    int n_extra = 0;
    const float* scale_a = nullptr;
    const float* scale_b = nullptr;
    uint32_t a_fmt = 0, b_fmt = 0;  // fp8 operand formats (0 = E4M3, 1 = E5M2)
};

template <int kKind, bool kAccF16, bool kBMn, int kBN, int kShape>
tcg_status launch_gemm(DeviceState& dev, const void* A, const void* B, void* C, int M, int N, int K,
                       int batches, cudaStream_t st, const EpiArgs& epi)
{
    void* const* extra = epi.extra;
    const int n_extra = epi.n_extra;
    constexpr bool kPair = kShape == kShapePair || kShape == kShapePairWide;
    // ring stages (int4 widens each stage in place: same depths as int8)
    constexpr int kStages = kShape == kShapeWide ? 3 : kShape == kShapePairWide ? 4
                            : kPair ? (kBN == 256 ? 6 : 8) : (kBN == 256 ? 4 : (kBN == 128 ? 6 : 8));
    constexpr bool kByte = kKind != kKindF16;
    using T = GemmTraits<kKind, kAccF16, kBMn, kBN, kStages, kShape>;
    auto kern = gemm_kernel<kKind, kAccF16, kBMn, kBN, kStages, kShape>;

    // the shared-memory opt-in once per kernel and device (not on every call,
    // which also keeps launches legal inside stream capture)
    static std::atomic<bool> smem_set[kMaxDevices];
    int dev_id = 0;
    cudaError_t e = cudaGetDevice(&dev_id);
    if (e != cudaSuccess) return cuda_fail(e);
    if (!smem_set[dev_id].load(std::memory_order_acquire)) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, T::kSmemBytes);
        if (e != cudaSuccess) return cuda_fail(e);
        smem_set[dev_id].store(true, std::memory_order_release);
    }

    const CUtensorMapDataType dt = kByte ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const uint64_t es = T::kElem;
    CUtensorMap mA, mB, mBh;  // mBh: B boxes of half the rows, for half tiles (K-major B)
    tcg_status s;
    if constexpr (kKind == kKindI4) {
        // packed operands (K / 2 bytes per row), 64-byte boxes (128 values of
        // K), unswizzled: the converter warps lay out the int8 stage
        const uint64_t kp = static_cast<uint64_t>(K) / 2;
        s = encode_3d(&mA, dt, A, kp, M, batches, kp, static_cast<uint64_t>(M) * kp, 64, kBM,
                      CU_TENSOR_MAP_SWIZZLE_NONE);
        if (s == TCG_SUCCESS)
            s = encode_3d(&mB, dt, B, kp, N, batches, kp, static_cast<uint64_t>(N) * kp, 64, T::kBRows,
                          CU_TENSOR_MAP_SWIZZLE_NONE);
        if (s == TCG_SUCCESS)
            s = encode_3d(&mBh, dt, B, kp, N, batches, kp, static_cast<uint64_t>(N) * kp, 64, T::kBRows / 2,
                          CU_TENSOR_MAP_SWIZZLE_NONE);
        if (s != TCG_SUCCESS) return s;
    } else {
    s = encode_3d(&mA, dt, A, K, M, batches, K * es, static_cast<uint64_t>(M) * K * es, T::kBK, kBM);
    if (s != TCG_SUCCESS) return s;
    if (kBMn) {  // B is K x N, N contiguous; half tiles load fewer 128-byte atoms
        s = encode_3d(&mB, dt, B, N, K, batches, N * es, static_cast<uint64_t>(K) * N * es, T::kAtomN, T::kBK);
        mBh = mB;
    } else {  // B is N x K, K contiguous
        s = encode_3d(&mB, dt, B, K, N, batches, K * es, static_cast<uint64_t>(N) * K * es, T::kBK, T::kBRows);
        if (s == TCG_SUCCESS)
            s = encode_3d(&mBh, dt, B, K, N, batches, K * es, static_cast<uint64_t>(N) * K * es, T::kBK,
                          T::kBRows / 2);
    }
    if (s != TCG_SUCCESS) return s;
    }

    GemmParams p;
    p.C = C;
    p.batch_stride_c = static_cast<long long>(M) * N;
    p.M = M;
    p.N = N;
    p.K = K;
    p.batches = batches;
    p.tiles_m = (M + T::kTileM - 1) / T::kTileM;
    p.tiles_n = (N + kBN - 1) / kBN;
    p.num_kb = (K + T::kBK - 1) / T::kBK;
    p.group_m = choose_group_m(T::kTileM, kBN, kPair ? dev.sms / 2 : dev.sms, p.tiles_m);
    static const int env_kalt = env_int("TCG_K_ALT", 1);
    p.k_alternate = ((kKind == kKindI8 || kKind == kKindI4) && env_kalt) ? 1 : 0;  // integer sums are order-free
    // Optional L2 eviction priorities for the A / B loads (-1 = no hint, the
    // default: on B200 the hinted loads doubled DRAM traffic at 32768^3).
    static const int env_l2a = env_int("TCG_L2_A", -1);
    static const int env_l2b = env_int("TCG_L2_B", -1);
    p.l2_a = env_l2a;
    p.l2_b = env_l2b;
    p.n_extra = n_extra;
    // instruction descriptors of a whole tile (N = kBN) and of a half tile
    const auto idesc_for = [&](int n) {
        if constexpr (kKind == kKindI8 || kKind == kKindI4)
            return make_idesc(2u, 1u, 1u, kBMn, T::kUmmaM, n);  // S32 <- s8 x s8
        else if constexpr (kKind == kKindF8)
            return make_idesc(1u, epi.a_fmt, epi.b_fmt, kBMn, T::kUmmaM, n);  // F32 <- e4m3/e5m2
        else
            return make_idesc(kAccF16 ? 0u : 1u, 0u, 0u, kBMn, T::kUmmaM, n);  // F32|F16 <- f16
    };
    p.idesc = idesc_for(kBN);
    p.idesc_half = idesc_for(kBN / 2);
    p.scale_a = epi.scale_a;
    p.scale_b = epi.scale_b;
    for (int i = 0; i < kMaxExtraDst; ++i) p.extra[i] = i < n_extra ? extra[i] : nullptr;
    p.vec_store = ((N % 4) == 0 && (reinterpret_cast<uintptr_t>(C) % 16) == 0) ? 1 : 0;
    for (int i = 0; i < n_extra; ++i)  // every destination must take 16-byte stores like C
        if ((reinterpret_cast<uintptr_t>(extra[i]) & 15u) != 0) p.vec_store = 0;
    // C through a tensor map (32 x 32 word boxes, 128-byte swizzle) when its
    // rows (and every peer destination) are 16-byte aligned; peer copies are
    // then plain stores from the same staging tile
    static const int env_tma_store = env_int("TCG_TMA_STORE", 1);
    p.tma_store = (env_tma_store && p.vec_store) ? 1 : 0;
    CUtensorMap mC;
    std::memset(&mC, 0, sizeof mC);
    if (p.tma_store) {
        s = encode_3d(&mC, CU_TENSOR_MAP_DATA_TYPE_INT32, C, N, M, batches, static_cast<uint64_t>(N) * 4,
                      static_cast<uint64_t>(M) * N * 4, 32, 32);
        if (s != TCG_SUCCESS) return s;
    }
    p.timeout_ns = g_timeout_ns.load();

    const long long tiles = static_cast<long long>(p.tiles_m) * p.tiles_n * batches;
    if (tiles > 0x3fffffffLL) return TCG_ERR_SHAPE;
    static const int env_units = env_int("TCG_UNITS");  // cap on persistent CTAs (pairs), tuning only
    static const int env_split = env_int("TCG_TAIL_SPLIT", 1);
    cudaLaunchConfig_t cfg;
    std::memset(&cfg, 0, sizeof cfg);
    cudaLaunchAttribute attr[2];
    std::memset(attr, 0, sizeof attr);
    cfg.blockDim = dim3(T::kThreadCount, 1, 1);
    cfg.dynamicSmemBytes = T::kSmemBytes;
    cfg.stream = st;
    cfg.attrs = attr;
    long long units = dev.sms;
    if constexpr (kPair) {
        const long long pairs = dev.sms / 2;
        cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs), 1, 1);
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.numAttrs = 1;
        // pairs resident at once: the wave size, and the grid of a static schedule
        static int max_clusters[kMaxDevices] = {0};
        if (max_clusters[dev_id] == 0) {
            int n = 0;
            if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
                cudaGetLastError();  // not fatal: fall back to one pair per two SMs
                n = static_cast<int>(pairs);
            }
            max_clusters[dev_id] = n;
        }
        units = max_clusters[dev_id] < pairs ? max_clusters[dev_id] : pairs;
    }
    if (env_units > 0 && env_units < units) units = env_units;
    // Tail split: when the last wave of tiles would leave at least half of the
    // units idle, its tiles are cut into column halves (two work items each),
    // which the idle units take; that wave then lasts about half as long.
    // Each half is an ordinary tile of N = kBN / 2: no cross-unit reduction,
    // and every output element is computed exactly as without the split.
    constexpr bool kCanSplit = !kBMn || (T::kBRows / 2) % T::kAtomN == 0;
    const long long rem = tiles % units;
    p.split_from = static_cast<int>(tiles);
    if (kCanSplit && env_split && rem > 0 && 2 * rem <= units) p.split_from = static_cast<int>(tiles - rem);
    const long long work = p.split_from + 2 * (tiles - p.split_from);
    // Scheduling.  Dynamic (the default whenever there is more than one wave
    // of work): one cluster (CTA) per work item; the clusters the GPU can hold
    // start, and each, when it finishes an item, takes over the next
    // not-yet-started cluster's item through cluster launch control -- in
    // launch order, so the items in flight stay a contiguous stretch of the
    // rasterised order however unevenly the units progress, and L2 keeps
    // serving the operand panels they share.  Static: one persistent unit per
    // resident slot, items round-robin.
    static const int env_static = env_int("TCG_STATIC_SCHEDULE");
    p.dynamic = (!env_static && work > units && (kPair ? 2 : 1) * work <= 0x7fffffffLL) ? 1 : 0;
    p.wave_units = static_cast<int>(units);
    // Stream-K (integer kinds, two-CTA 512 x 256 tiles, one to four waves
    // with a partial last one): every resident pair takes an equal share of
    // the tiles' k-blocks laid end to end, so the last wave is not mostly
    // idle.  A tile cut between two pairs: the pair with its first k-blocks
    // (the head, its first item) stores its partial sums into C as usual and
    // flags them; the pair with the rest (the tail, its last item) adds its
    // sums onto them with TMA reduce-add stores.  Exact for integers; the
    // floating-point kinds keep one k order per element and are not split.
    // Static schedule (one persistent cluster per pair, all resident).
    // Opt-in (TCG_STREAM_K=1): measured on B200 it loses to the data-parallel
    // schedule at every shape tried -- the mainloop is bound by operand
    // delivery (~0.8 us per k-block of a 512 x 256 tile with 74 pairs
    // streaming), so giving the idle pairs of a partial wave work does not
    // shorten the critical path, and the extra item boundary costs a drain.
    p.sk = 0;
    p.sk_units = 0;
    p.sk_work = 0;
    p.sk_epoch = 0;
    p.sk_slot = 0;
    static const int env_sk = env_int("TCG_STREAM_K", 0);
    if constexpr (kShape == kShapePairWide) {
        const double waves = static_cast<double>(tiles) / static_cast<double>(units);
        const double rounds = static_cast<double>((tiles + units - 1) / units);
        if ((kKind == kKindI8 || kKind == kKindI4) && epi.scale_a == nullptr && p.tma_store && env_sk &&
            n_extra == 0 && tiles > units && tiles <= 4 * units && tiles % units != 0 &&
            waves < 0.95 * rounds && p.num_kb >= 4 && units <= kSkMaxUnits) {
            static std::atomic<unsigned int> epoch{0};
            unsigned int e = ++epoch;
            if (e == 0) e = ++epoch;  // 0 marks a consumed flag
            p.sk = 1;
            p.sk_units = static_cast<int>(units);
            p.sk_work = tiles * p.num_kb;
            p.sk_epoch = e;
            p.sk_slot = static_cast<int>(e % kSkSlots);
            p.split_from = static_cast<int>(tiles);
            p.k_alternate = 0;
            p.dynamic = 0;
        }
    }
    const long long grid_units = p.sk ? units : p.dynamic ? work : (work < units ? work : units);
    static const int debug = env_int("TCG_DEBUG");
    if (debug)
        std::fprintf(stderr, "tcgemm: %s tile %dx%d stages %d units %lld grid %lld tiles %lld split_from %d group_m %d kalt %d %s\n",
                     kPair ? "pair" : (T::kWide ? "wide" : "single"), T::kTileM, kBN, kStages, units,
                     grid_units, tiles, p.split_from, p.group_m, p.k_alternate,
                     p.sk ? "stream-k" : p.dynamic ? "dynamic" : "static");
    // Programmatic dependent launch: this grid may start while the previous
    // kernel on the stream finishes; it waits (griddepcontrol.wait) before
    // touching global memory.
    if (pdl_enabled()) {
        attr[cfg.numAttrs].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[cfg.numAttrs].val.programmaticStreamSerializationAllowed = 1;
        ++cfg.numAttrs;
    }
    cfg.gridDim = dim3(static_cast<unsigned>((kPair ? 2 : 1) * grid_units), 1, 1);
    e = cudaLaunchKernelEx(&cfg, kern, mA, mB, mBh, mC, p);
    if (e != cudaSuccess) return cuda_fail(e);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e);
    t_last_tile_n = kBN;
    t_last_tile_m = T::kTileM;
    return TCG_SUCCESS;
}

template <int kKind, bool kAccF16, bool kBMn>
tcg_status dispatch_bn(DeviceState& dev, const void* A, const void* B, void* C, int M, int N, int K,
                       int batches, cudaStream_t st, const EpiArgs& epi = EpiArgs())
{
    constexpr bool kByteMn = kKind != kKindF16 && kBMn;  // MN-major byte operand: 128-column atoms
    const TileChoice c = choose_tile(M, N, K, kKind == kKindF16 ? 2 : 1, batches, dev.sms, kByteMn);
    if (c.shape == kShapeWide) return launch_gemm<kKind, kAccF16, kBMn, 256, kShapeWide>(dev, A, B, C, M, N, K, batches, st, epi);
    if (c.shape == kShapePairWide)
        return launch_gemm<kKind, kAccF16, kBMn, 256, kShapePairWide>(dev, A, B, C, M, N, K, batches, st, epi);
    if (c.shape == kShapePair) {
        if (c.bn == 128) {
            // an MN-major byte pair tile needs 128 columns per CTA
            if constexpr (!kByteMn) return launch_gemm<kKind, kAccF16, kBMn, 128, kShapePair>(dev, A, B, C, M, N, K, batches, st, epi);
        }
        return launch_gemm<kKind, kAccF16, kBMn, 256, kShapePair>(dev, A, B, C, M, N, K, batches, st, epi);
    }
    switch (c.bn) {
    case 64:
        if constexpr (!kByteMn) return launch_gemm<kKind, kAccF16, kBMn, 64, kShapeSingle>(dev, A, B, C, M, N, K, batches, st, epi);
        [[fallthrough]];
    case 128: return launch_gemm<kKind, kAccF16, kBMn, 128, kShapeSingle>(dev, A, B, C, M, N, K, batches, st, epi);
    default: return launch_gemm<kKind, kAccF16, kBMn, 256, kShapeSingle>(dev, A, B, C, M, N, K, batches, st, epi);
    }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
bool aligned4(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 3u) == 0; }

// Shared validation; returns TCG_SUCCESS with *done = true when there is no
// work left (empty problem, or K == 0 handled by zero-filling C).
tcg_status prologue(const void* A, const void* B, void* C, int M, int N, int K, int batches, cudaStream_t st,
                    bool* done)
{
    *done = false;
    if (M < 0 || N < 0 || K < 0 || batches < 0) return TCG_ERR_SHAPE;
    if (M == 0 || N == 0 || batches == 0) {
        *done = true;
        return TCG_SUCCESS;
    }
    if (!C) return TCG_ERR_ARG;
    if (!aligned4(C)) return TCG_ERR_ALIGN;
    if (K == 0) {
        cudaError_t e = cudaMemsetAsync(C, 0, static_cast<size_t>(M) * N * batches * 4, st);
        if (e != cudaSuccess) return cuda_fail(e);
        *done = true;
        return TCG_SUCCESS;
    }
    if (!A || !B) return TCG_ERR_ARG;
    if (!aligned16(A) || !aligned16(B)) return TCG_ERR_ALIGN;
    return TCG_SUCCESS;
}

size_t round256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

UnpackSeg unpack_seg(const int8_t* in, int8_t* out, size_t n_packed)
{
    UnpackSeg g;
    g.n16 = static_cast<long long>(n_packed / 16);
    g.in = reinterpret_cast<const uint4*>(in);
    g.out = reinterpret_cast<uint4*>(out);
    g.tail_in = in + g.n16 * 16;
    g.tail_out = out + g.n16 * 32;
    g.tail = static_cast<int>(n_packed % 16);
    return g;
}

// Widen one or two packed int4 tensors (n1 = 0: one) in a single launch.
tcg_status launch_unpack(const int8_t* in0, int8_t* out0, size_t n0, const int8_t* in1, int8_t* out1, size_t n1,
                         int sms, cudaStream_t st)
{
    const UnpackSeg s0 = unpack_seg(in0, out0, n0);
    const UnpackSeg s1 = n1 ? unpack_seg(in1, out1, n1) : unpack_seg(in0, out0, 0);
    const long long chunks = s0.n16 + s1.n16;
    long long blocks = (chunks + 1023) / 1024;  // four chunks per thread
    const long long cap = static_cast<long long>(sms) * 8;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    cudaLaunchConfig_t cfg;
    std::memset(&cfg, 0, sizeof cfg);
    cudaLaunchAttribute attr[1];
    std::memset(attr, 0, sizeof attr);
    cfg.gridDim = dim3(static_cast<unsigned>(blocks), 1, 1);
    cfg.blockDim = dim3(256, 1, 1);
    cfg.stream = st;
    cfg.attrs = attr;
    if (pdl_enabled()) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.numAttrs = 1;
    }
    cudaError_t e = cudaLaunchKernelEx(&cfg, unpack_s4_kernel, s0, s1);
    return e == cudaSuccess ? TCG_SUCCESS : cuda_fail(e);
}

}  // namespace

extern "C" {

tcg_status tcg_gemm_f16(const void* A, const void* B, float* C, int M, int N, int K, int batches, tcg_acc acc,
                        tcg_b_layout b_layout, void* stream)
{
    if (acc != TCG_ACC_F32 && acc != TCG_ACC_F16) return TCG_ERR_ARG;
    if (b_layout != TCG_B_KN && b_layout != TCG_B_NK) return TCG_ERR_ARG;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    bool done;
    tcg_status s = prologue(A, B, C, M, N, K, batches, st, &done);
    if (s != TCG_SUCCESS || done) return s;
    if (K % 8 != 0) return TCG_ERR_SHAPE;
    if (b_layout == TCG_B_KN && N % 8 != 0) return TCG_ERR_SHAPE;
    DeviceState* dev;
    if ((s = device_state(&dev)) != TCG_SUCCESS) return s;
    if ((s = resolve_encode()) != TCG_SUCCESS) return s;
    if (acc == TCG_ACC_F32)
        return b_layout == TCG_B_KN ? dispatch_bn<kKindF16, false, true>(*dev, A, B, C, M, N, K, batches, st)
                                    : dispatch_bn<kKindF16, false, false>(*dev, A, B, C, M, N, K, batches, st);
    return b_layout == TCG_B_KN ? dispatch_bn<kKindF16, true, true>(*dev, A, B, C, M, N, K, batches, st)
                                : dispatch_bn<kKindF16, true, false>(*dev, A, B, C, M, N, K, batches, st);
}

tcg_status tcg_gemm_s8(const int8_t* A, const int8_t* B, int32_t* C, int M, int N, int K, int batches,
                       tcg_b_layout b_layout, void* stream)
{
    if (b_layout != TCG_B_KN && b_layout != TCG_B_NK) return TCG_ERR_ARG;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    bool done;
    tcg_status s = prologue(A, B, C, M, N, K, batches, st, &done);
    if (s != TCG_SUCCESS || done) return s;
    if (K % 16 != 0) return TCG_ERR_SHAPE;
    if (b_layout == TCG_B_KN && N % 16 != 0) return TCG_ERR_SHAPE;
    DeviceState* dev;
    if ((s = device_state(&dev)) != TCG_SUCCESS) return s;
    if ((s = resolve_encode()) != TCG_SUCCESS) return s;
    return b_layout == TCG_B_KN ? dispatch_bn<kKindI8, false, true>(*dev, A, B, C, M, N, K, batches, st)
                                : dispatch_bn<kKindI8, false, false>(*dev, A, B, C, M, N, K, batches, st);
}

tcg_status tcg_gemm_s8_multi(const int8_t* A, const int8_t* B, int32_t* const* C_dst, int n_dst, int M, int N,
                             int K, tcg_b_layout b_layout, void* stream)
{
    if (b_layout != TCG_B_KN && b_layout != TCG_B_NK) return TCG_ERR_ARG;
    if (!C_dst || n_dst < 1 || n_dst > 1 + kMaxExtraDst) return TCG_ERR_ARG;
    for (int i = 0; i < n_dst; ++i)
        if (!C_dst[i]) return TCG_ERR_ARG;
        else if (!aligned4(C_dst[i])) return TCG_ERR_ALIGN;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    bool done;
    tcg_status s = prologue(A, B, C_dst[0], M, N, K, 1, st, &done);
    if (s != TCG_SUCCESS) return s;
    if (done) {
        if (M > 0 && N > 0 && K == 0)  // zero-fill every destination, as for C
            for (int i = 1; i < n_dst; ++i) {
                cudaError_t e = cudaMemsetAsync(C_dst[i], 0, static_cast<size_t>(M) * N * 4, st);
                if (e != cudaSuccess) return cuda_fail(e);
            }
        return TCG_SUCCESS;
    }
    if (K % 16 != 0) return TCG_ERR_SHAPE;
    if (b_layout == TCG_B_KN && N % 16 != 0) return TCG_ERR_SHAPE;
    DeviceState* dev;
    if ((s = device_state(&dev)) != TCG_SUCCESS) return s;
    if ((s = resolve_encode()) != TCG_SUCCESS) return s;
    EpiArgs epi;
    epi.extra = reinterpret_cast<void* const*>(C_dst + 1);
    epi.n_extra = n_dst - 1;
    return b_layout == TCG_B_KN ? dispatch_bn<kKindI8, false, true>(*dev, A, B, C_dst[0], M, N, K, 1, st, epi)
                                : dispatch_bn<kKindI8, false, false>(*dev, A, B, C_dst[0], M, N, K, 1, st, epi);
}

tcg_status tcg_gemm_f8(const void* A, const void* B, float* C, int M, int N, int K, int batches,
                       tcg_f8_format a_fmt, tcg_f8_format b_fmt, tcg_b_layout b_layout, void* stream)
{
    if (b_layout != TCG_B_KN && b_layout != TCG_B_NK) return TCG_ERR_ARG;
    if ((a_fmt != TCG_F8_E4M3 && a_fmt != TCG_F8_E5M2) || (b_fmt != TCG_F8_E4M3 && b_fmt != TCG_F8_E5M2))
        return TCG_ERR_ARG;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    bool done;
    tcg_status s = prologue(A, B, C, M, N, K, batches, st, &done);
    if (s != TCG_SUCCESS || done) return s;
    if (K % 16 != 0) return TCG_ERR_SHAPE;
    if (b_layout == TCG_B_KN && N % 16 != 0) return TCG_ERR_SHAPE;
    DeviceState* dev;
    if ((s = device_state(&dev)) != TCG_SUCCESS) return s;
    if ((s = resolve_encode()) != TCG_SUCCESS) return s;
    EpiArgs epi;
    epi.a_fmt = static_cast<uint32_t>(a_fmt);
    epi.b_fmt = static_cast<uint32_t>(b_fmt);
    return b_layout == TCG_B_KN ? dispatch_bn<kKindF8, false, true>(*dev, A, B, C, M, N, K, batches, st, epi)
                                : dispatch_bn<kKindF8, false, false>(*dev, A, B, C, M, N, K, batches, st, epi);
}

size_t tcg_gemm_s4_workspace_size(int M, int N, int K, int batches)
{
    if (M <= 0 || N <= 0 || K <= 0 || batches <= 0) return 0;
    return round256(static_cast<size_t>(batches) * M * K) + round256(static_cast<size_t>(batches) * N * K);
}

}  // extern "C"

namespace {

// int4 in two passes: both operands widened into scratch (A then B, 256-byte
// aligned) by unpack_s4_kernel, then the int8 GEMM.  The scratch is the
// caller's `workspace`, or, when that is NULL, a stream-ordered allocation
// from the device's private pool.  tcg_gemm_s4_static runs this form with its
// fixed device array; TCG_S4_PREPASS=1 selects it for tcg_gemm_s4 too.
tcg_status gemm_s4_prepass(const int8_t* A_packed, const int8_t* BT_packed, void* C, int M, int N, int K,
                           int batches, void* workspace, size_t workspace_bytes, cudaStream_t st,
                           const EpiArgs& epi, DeviceState* dev)
{
    tcg_status s;
    const size_t need = tcg_gemm_s4_workspace_size(M, N, K, batches);
    void* ws = workspace;
    bool owned = false;
    if (ws) {
        if (workspace_bytes < need) return TCG_ERR_WORKSPACE;
        if (reinterpret_cast<uintptr_t>(ws) & 255u) return TCG_ERR_ALIGN;
    } else {
        std::lock_guard<std::mutex> lk(dev->mu);
        if (!dev->pool) {
            int d = 0;
            cudaGetDevice(&d);
            cudaMemPoolProps props;
            std::memset(&props, 0, sizeof props);
            props.allocType = cudaMemAllocationTypePinned;
            props.location.type = cudaMemLocationTypeDevice;
            props.location.id = d;
            cudaError_t e = cudaMemPoolCreate(&dev->pool, &props);
            if (e != cudaSuccess) return cuda_fail(e);
            unsigned long long keep = ~0ull;  // keep freed blocks for the next call
            cudaMemPoolSetAttribute(dev->pool, cudaMemPoolAttrReleaseThreshold, &keep);
        }
        cudaError_t e = cudaMallocFromPoolAsync(&ws, need, dev->pool, st);
        if (e != cudaSuccess) return cuda_fail(e);
        owned = true;
    }
    int8_t* a8 = static_cast<int8_t*>(ws);
    int8_t* b8 = a8 + round256(static_cast<size_t>(batches) * M * K);
    s = launch_unpack(A_packed, a8, static_cast<size_t>(batches) * M * (K / 2), BT_packed, b8,
                      static_cast<size_t>(batches) * N * (K / 2), dev->sms, st);
    if (s == TCG_SUCCESS) s = dispatch_bn<kKindI8, false, false>(*dev, a8, b8, C, M, N, K, batches, st, epi);
    if (owned) {
        cudaError_t e = cudaFreeAsync(ws, st);
        if (e != cudaSuccess && s == TCG_SUCCESS) s = cuda_fail(e);
    }
    return s;
}

// Validation shared by the int4 entries; *dev set when there is work.
tcg_status s4_prologue(const int8_t* A_packed, const int8_t* BT_packed, void* C, int M, int N, int K, int batches,
                       cudaStream_t st, bool* done, DeviceState** dev)
{
    tcg_status s = prologue(A_packed, BT_packed, C, M, N, K, batches, st, done);
    if (s != TCG_SUCCESS || *done) return s;
    if (K % 32 != 0) return TCG_ERR_SHAPE;
    if ((s = device_state(dev)) != TCG_SUCCESS) return s;
    return resolve_encode();
}

// int4 GEMM.  By default one fused kernel: TMA brings the packed operands
// into a staging ring and converter warps widen them to int8 in shared
// memory, next to the MMAs -- no scratch, no allocation, no second pass over
// HBM.  The workspace arguments only matter for the two-pass form.
tcg_status gemm_s4_impl(const int8_t* A_packed, const int8_t* BT_packed, void* C, int M, int N, int K, int batches,
                        void* workspace, size_t workspace_bytes, void* stream, const EpiArgs& epi)
{
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    bool done;
    DeviceState* dev = nullptr;
    tcg_status s = s4_prologue(A_packed, BT_packed, C, M, N, K, batches, st, &done, &dev);
    if (s != TCG_SUCCESS || done) return s;
    // the fused kernel's accumulators hold 256 x the result: K < 2^17 keeps
    // them in int32; longer K takes the two-pass form
    static const int env_prepass = env_int("TCG_S4_PREPASS");
    if (env_prepass || K >= (1 << 17))
        return gemm_s4_prepass(A_packed, BT_packed, C, M, N, K, batches, workspace, workspace_bytes, st, epi, dev);
    return dispatch_bn<kKindI4, false, false>(*dev, A_packed, BT_packed, C, M, N, K, batches, st, epi);
}

}  // namespace

extern "C" {

tcg_status tcg_gemm_s4(const int8_t* A_packed, const int8_t* BT_packed, int32_t* C, int M, int N, int K,
                       int batches, void* workspace, size_t workspace_bytes, void* stream)
{
    return gemm_s4_impl(A_packed, BT_packed, C, M, N, K, batches, workspace, workspace_bytes, stream, EpiArgs());
}

tcg_status tcg_gemm_s4_dequant(const int8_t* A_packed, const int8_t* BT_packed, float* C, int M, int N, int K,
                               int batches, const float* scale_a, const float* scale_b, void* workspace,
                               size_t workspace_bytes, void* stream)
{
    if (!scale_a || !scale_b) return TCG_ERR_ARG;
    EpiArgs epi;
    epi.scale_a = scale_a;
    epi.scale_b = scale_b;
    return gemm_s4_impl(A_packed, BT_packed, C, M, N, K, batches, workspace, workspace_bytes, stream, epi);
}

tcg_status tcg_gemm_s8_dequant(const int8_t* A, const int8_t* B, float* C, int M, int N, int K, int batches,
                               tcg_b_layout b_layout, const float* scale_a, const float* scale_b, void* stream)
{
    if (b_layout != TCG_B_KN && b_layout != TCG_B_NK) return TCG_ERR_ARG;
    if (!scale_a || !scale_b) return TCG_ERR_ARG;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    bool done;
    tcg_status s = prologue(A, B, C, M, N, K, batches, st, &done);
    if (s != TCG_SUCCESS || done) return s;
    if (K % 16 != 0) return TCG_ERR_SHAPE;
    if (b_layout == TCG_B_KN && N % 16 != 0) return TCG_ERR_SHAPE;
    DeviceState* dev;
    if ((s = device_state(&dev)) != TCG_SUCCESS) return s;
    if ((s = resolve_encode()) != TCG_SUCCESS) return s;
    EpiArgs epi;
    epi.scale_a = scale_a;
    epi.scale_b = scale_b;
    return b_layout == TCG_B_KN ? dispatch_bn<kKindI8, false, true>(*dev, A, B, C, M, N, K, batches, st, epi)
                                : dispatch_bn<kKindI8, false, false>(*dev, A, B, C, M, N, K, batches, st, epi);
}

static tcg_status quantize_common(const float* src, int8_t* dst, long long n, long long n_out_units, bool s4,
                                  float* scale, void* stream)
{
    if (n == 0) return TCG_SUCCESS;
    if (!src || !dst || !scale) return TCG_ERR_ARG;
    if ((reinterpret_cast<uintptr_t>(src) & 15u) || (reinterpret_cast<uintptr_t>(dst) & 3u) ||
        (reinterpret_cast<uintptr_t>(scale) & 3u))
        return TCG_ERR_ALIGN;
    DeviceState* dev;
    tcg_status s = device_state(&dev);
    if (s != TCG_SUCCESS) return s;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemsetAsync(scale, 0, sizeof(float), st);
    if (e != cudaSuccess) return cuda_fail(e);
    const long long cap = static_cast<long long>(dev->sms) * 8;
    long long blocks = (n / 4 + 255) / 256;
    blocks = blocks < 1 ? 1 : (blocks > cap ? cap : blocks);
    absmax_kernel<<<static_cast<int>(blocks), 256, 0, st>>>(src, n, reinterpret_cast<int*>(scale));
    long long qblocks = (n_out_units + 255) / 256;
    qblocks = qblocks < 1 ? 1 : (qblocks > cap ? cap : qblocks);
    if (s4)
        quantize_s4_kernel<<<static_cast<int>(qblocks), 256, 0, st>>>(src, dst, n_out_units,
                                                                      reinterpret_cast<const int*>(scale));
    else
        quantize_s8_kernel<<<static_cast<int>(qblocks), 256, 0, st>>>(src, dst, n,
                                                                      reinterpret_cast<const int*>(scale));
    publish_scale_kernel<<<1, 1, 0, st>>>(scale, s4 ? 7.f : 127.f);
    e = cudaGetLastError();
    return e == cudaSuccess ? TCG_SUCCESS : cuda_fail(e);
}

tcg_status tcg_quantize_absmax_s8(const float* src, int8_t* dst, size_t n, float* scale, void* stream)
{
    return quantize_common(src, dst, static_cast<long long>(n), static_cast<long long>(n) / 4, false, scale, stream);
}

tcg_status tcg_quantize_absmax_s4(const float* src, int8_t* dst_packed, int rows, int cols_k, float* scale,
                                  void* stream)
{
    if (rows < 0 || cols_k < 0 || (cols_k & 1)) return TCG_ERR_SHAPE;
    const long long n = static_cast<long long>(rows) * cols_k;
    return quantize_common(src, dst_packed, n, n / 2, true, scale, stream);
}

}  // extern "C"

// ---- int4 GEMM without allocation: scratch in a fixed device array -------
//
// For callers that may not allocate device memory (see tcgemm.h).  Host code
// must never pass `g_s4_static_scratch` itself to a kernel: on the host that
// name is only a stand-in for the symbol, not a device address.  The device
// address is looked up once per device with cudaGetSymbolAddress.
namespace {

static __device__ __align__(256) unsigned char g_s4_static_scratch[TCG_S4_STATIC_SCRATCH_BYTES];

struct StaticScratch {
    std::mutex mu;
    void* ptr = nullptr;  // set once a lookup has succeeded
};
StaticScratch g_s4_static[kMaxDevices];

// Device address of the array on the current device.  The lookup runs with
// that device current, on the first call per device; only a successful
// lookup is kept, so a call that failed (inside a stream capture, say) is
// retried by the next one.  cudaDeviceReset is not supported while the
// library is in use: it unloads the module that holds the array.
tcg_status static_scratch(void** out)
{
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e);
    if (dev < 0 || dev >= kMaxDevices) return TCG_ERR_UNSUPPORTED;
    StaticScratch& s = g_s4_static[dev];
    std::lock_guard<std::mutex> lk(s.mu);
    if (!s.ptr) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_s4_static_scratch);
        if (e != cudaSuccess) return cuda_fail(e);
        if (!p) return cuda_fail(cudaErrorInvalidSymbol);
        s.ptr = p;
    }
    *out = s.ptr;
    return TCG_SUCCESS;
}

}  // namespace

extern "C" {

tcg_status tcg_gemm_s4_static(const int8_t* A_packed, const int8_t* BT_packed, int32_t* C, int M, int N, int K,
                              int batches, void* stream)
{
    if (M < 0 || N < 0 || K < 0 || batches < 0) return TCG_ERR_SHAPE;
    if (tcg_gemm_s4_workspace_size(M, N, K, batches) > TCG_S4_STATIC_SCRATCH_BYTES) return TCG_ERR_WORKSPACE;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    bool done;
    DeviceState* dev = nullptr;
    tcg_status s = s4_prologue(A_packed, BT_packed, C, M, N, K, batches, st, &done, &dev);
    if (s != TCG_SUCCESS || done) return s;
    void* ws = nullptr;
    if ((s = static_scratch(&ws)) != TCG_SUCCESS) return s;
    // the two-pass form with the fixed array as its scratch: nothing is allocated
    return gemm_s4_prepass(A_packed, BT_packed, C, M, N, K, batches, ws, TCG_S4_STATIC_SCRATCH_BYTES, st,
                           EpiArgs(), dev);
}

tcg_status tcg_unpack_s4(const int8_t* packed, int8_t* out, size_t n_packed, void* stream)
{
    if (n_packed == 0) return TCG_SUCCESS;
    if (!packed || !out) return TCG_ERR_ARG;
    if (!aligned16(packed) || !aligned16(out)) return TCG_ERR_ALIGN;
    DeviceState* dev;
    tcg_status s = device_state(&dev);
    if (s != TCG_SUCCESS) return s;
    return launch_unpack(packed, out, n_packed, nullptr, nullptr, 0, dev->sms, static_cast<cudaStream_t>(stream));
}

tcg_status tcg_check_device_error(void* stream, uint64_t* word)
{
    cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e);
    unsigned long long w = 0;
    e = cudaMemcpyFromSymbol(&w, tcg::g_tcg_error_word, sizeof w);
    if (e != cudaSuccess) return cuda_fail(e);
    if (word) *word = w;
    if (w == 0) return TCG_SUCCESS;
    const unsigned long long zero = 0;
    e = cudaMemcpyToSymbol(tcg::g_tcg_error_word, &zero, sizeof zero);
    if (e != cudaSuccess) return cuda_fail(e);
    return TCG_ERR_TIMEOUT;
}

tcg_status tcg_ipc_handle(const void* ptr, void* handle, size_t* offset)
{
    if (!ptr || !handle || !offset) return TCG_ERR_ARG;
    typedef CUresult (*RangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);
    static RangeFn range = nullptr;
    static std::once_flag once;
    std::call_once(once, []() {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            range = reinterpret_cast<RangeFn>(fn);
    });
    if (!range) return TCG_ERR_CUDA;
    CUdeviceptr base = 0;
    size_t size = 0;
    CUresult r = range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr));
    if (r != CUDA_SUCCESS) {
        t_last_cuda_error = static_cast<int>(r);
        return TCG_ERR_CUDA;
    }
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
    if (e != cudaSuccess) return cuda_fail(e);
    std::memcpy(handle, &h, sizeof h);
    *offset = reinterpret_cast<uintptr_t>(ptr) - static_cast<uintptr_t>(base);
    return TCG_SUCCESS;
}

tcg_status tcg_ipc_open(const void* handle, void** base)
{
    if (!handle || !base) return TCG_ERR_ARG;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof h);
    cudaError_t e = cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess);
    return e == cudaSuccess ? TCG_SUCCESS : cuda_fail(e);
}

tcg_status tcg_ipc_close(void* base)
{
    cudaError_t e = cudaIpcCloseMemHandle(base);
    return e == cudaSuccess ? TCG_SUCCESS : cuda_fail(e);
}

tcg_status tcg_copy_2d_async(void* dst, size_t dpitch, const void* src, size_t spitch, size_t width_bytes,
                             size_t height, void* stream)
{
    if (height == 0 || width_bytes == 0) return TCG_SUCCESS;
    if (!dst || !src || dpitch < width_bytes || spitch < width_bytes) return TCG_ERR_ARG;
    cudaError_t e = cudaMemcpy2DAsync(dst, dpitch, src, spitch, width_bytes, height, cudaMemcpyDefault,
                                      static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? TCG_SUCCESS : cuda_fail(e);
}

tcg_status tcg_host_register(void* ptr, size_t bytes)
{
    if (!ptr || bytes == 0) return TCG_ERR_ARG;
    cudaError_t e = cudaHostRegister(ptr, bytes, cudaHostRegisterPortable);
    return e == cudaSuccess ? TCG_SUCCESS : cuda_fail(e);
}

tcg_status tcg_host_unregister(void* ptr)
{
    if (!ptr) return TCG_ERR_ARG;
    cudaError_t e = cudaHostUnregister(ptr);
    return e == cudaSuccess ? TCG_SUCCESS : cuda_fail(e);
}

tcg_status tcg_selftest_wait_timeout(uint64_t timeout_ns, void* stream)
{
    DeviceState* dev;
    tcg_status s = device_state(&dev);
    if (s != TCG_SUCCESS) return s;
    wait_selftest_kernel<<<1, 64, 0, static_cast<cudaStream_t>(stream)>>>(timeout_ns);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? TCG_SUCCESS : cuda_fail(e);
}

void tcg_set_wait_timeout_ns(uint64_t ns) { g_timeout_ns.store(ns ? ns : 2000000000ull); }
void tcg_set_tile_n(int bn) { g_force_bn.store(bn); }
int tcg_last_cuda_error(void) { return t_last_cuda_error; }
int tcg_last_tile_n(void) { return t_last_tile_n; }
int tcg_last_tile_m(void) { return t_last_tile_m; }
void tcg_set_cta_pair(int mode) { g_force_pair.store(mode); }
int tcg_version(void) { return 100; }

const char* tcg_status_string(tcg_status s)
{
    switch (s) {
    case TCG_SUCCESS: return "success";
    case TCG_ERR_SHAPE: return "unsupported shape (see tcgemm.h shape rules)";
    case TCG_ERR_ALIGN: return "misaligned pointer (A/B need 16 bytes, C 4 bytes)";
    case TCG_ERR_TIMEOUT: return "a device-side wait timed out";
    case TCG_ERR_CUDA: return "CUDA runtime error";
    case TCG_ERR_ARG: return "invalid argument";
    case TCG_ERR_UNSUPPORTED: return "device is not sm_100 (B200)";
    case TCG_ERR_WORKSPACE: return "workspace too small";
    }
    return "unknown status";
}

}  // extern "C"
