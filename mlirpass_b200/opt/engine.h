// engine.h — the device side of dcfold-opt: constant residency on a GPU and
// execution of element-level fold requests through libdcfold's C ABI.
//
// Constants live where they are cheapest to use next.  A constant parsed
// from `dense<"0x…">` text is uploaded as text on first use and decoded on
// the device (dcf_hex_decode_async); a fold result stays on the device
// until the printer (or a host-side shortcut) needs it, so a chain of folds
// never round-trips through the host.  Results that come out all-equal are
// kept as one host-side element, as MLIR stores a splat.
#pragma once

#include "cuda_rt.h"

#include <memory>
#include <string>
#include <vector>

#include "../../include/dcfold.h"
#include "ir.h"

namespace dco {

// Device memory from a per-device caching pool: freed buffers are kept by
// size class and handed out again, so a fold chain reuses the same HBM
// instead of calling cudaMalloc / cudaFree for every intermediate.
class DeviceBuf {
 public:
  DeviceBuf(int device, size_t bytes);
  // A view of `bytes` bytes at `offset` inside `parent` (which it keeps
  // alive): the constants of one packed upload share their arena.
  DeviceBuf(std::shared_ptr<DeviceBuf> parent, size_t offset, size_t bytes);
  ~DeviceBuf();
  DeviceBuf(const DeviceBuf&) = delete;
  DeviceBuf& operator=(const DeviceBuf&) = delete;
  void* ptr = nullptr;
  size_t bytes = 0;
  size_t cap = 0;
  int device = 0;

 private:
  std::shared_ptr<DeviceBuf> parent_;
};

// One element-level fold.  The greedy driver fills the inputs; the engine
// fills the outcome.
struct FoldRequest {
  enum Kind { BINARY, CONVERT, RECIPROCAL, PERMUTE, SPLAT_SCAN, SELECT } kind = BINARY;
  int op = 0, dtype = 0, out_dtype = 0;
  uint32_t flags = 0;
  DenseP lhs, rhs;
  DenseP cond;                          // SELECT: i1 conditions; lhs / rhs are the values
  uint64_t n = 0;                       // result elements
  std::vector<int64_t> shape, perms;    // PERMUTE
  TypeP out_ty;                         // attribute type of the result
  bool out_elements = true;
  // A second result over the same operands (the *_extended ops): a second
  // binary kernel `op2` writing out2_dtype elements of type out2_ty.
  int op2 = 0, out2_dtype = 0;
  uint32_t flags2 = 0;
  TypeP out2_ty;
  DenseP out2;
  // outcome
  bool folded = false;
  uint64_t first_fail = ~0ull;
  DenseP out;
};

// One constant's bytes inside a packed transfer image: many constants
// travel through the pinned slots back to back, each at a 16-byte aligned
// offset of the image.
struct ImagePiece {
  void* host;         // source (upload) or destination (download)
  const void* dev;    // device source of a download
  size_t len, off;    // bytes, offset in the image
  bool hex = false;   // upload: `host` is hex text of 2 * len characters, decoded on the way
};

// Decode `nbytes` bytes from 2 * nbytes hex characters (either case) on the
// host; false if any character is not a hex digit.  Thread-safe.
bool decode_hex_host(const char* in, size_t nbytes, uint8_t* out);

struct EngineStats {
  uint64_t h2d_bytes = 0, d2h_bytes = 0, requests = 0, batches = 0;
  double device_ms = 0;    // sum of batch wall times
  double upload_ms = 0;    // to_device_all: staging, copies, decode
  double download_ms = 0;  // to_host_all
};

// device < 0 makes a host-only engine: parsing, printing and the folds that
// the host decides alone (shortcuts) work, and any element work throws.
class Engine {
 public:
  explicit Engine(int device);
  virtual ~Engine();
  virtual int device() const { return dev_; }

  // Run every request (all belong to this engine's device).  Throws on a
  // runtime error; a refused fold is an outcome, not an error.
  virtual void execute(const std::vector<FoldRequest*>& reqs);

  // Make a constant resident on this device.
  virtual void to_device(DenseValue& v);
  // Make its bytes available on the host (downloading if needed).
  virtual void to_host(DenseValue& v);
  // The same for many constants with one synchronisation: their hex texts
  // (or host bytes) are packed back to back through the pinned slots into
  // one device arena and decoded there; results come back through the
  // slots the same way.
  virtual void to_device_all(const std::vector<DenseValue*>& vs);
  virtual void to_host_all(const std::vector<DenseValue*>& vs);
  // Uppercase hex digits of all its bytes (encoded on the device when
  // the value is there).
  virtual std::string hex_of(DenseValue& v);
  virtual uint64_t bits0_of(DenseValue& v);
  // 64-bit hash of the bytes (dcf_hash_many_async; computed on upload and
  // for every fold result, so deduplication rarely launches anything).
  virtual uint64_t hash_of(DenseValue& v);
  // Whether every value equals the first (cached in v.all_equal).
  virtual bool all_equal(DenseValue& v);

  EngineStats stats;

  // Host memory the copy engine can read directly (page-locked input
  // text): its literals are copied straight from there as text and decoded
  // on the GPU, with no host core touching them.  With small_on_host (one
  // GPU in the run), literals of less than kSmallPinnedHex characters are
  // decoded by the host threads instead, as pageable text is: measured on
  // one B200, config 5's 8192 literals of 512 KB ran 183 ms that way
  // against 216 ms, while config 2's 134 MB literals ran 12.6 ms on the
  // device against 16.1 ms; with several GPUs decoding on the host for all
  // of them was CPU-bound (config 5 at 8 GPUs: 103 against 64 ms).
  static constexpr size_t kSmallPinnedHex = 4u << 20;
  void set_pinned_source(const void* begin, size_t bytes, bool small_on_host) {
    pinned_src_ = (const char*)begin;
    pinned_len_ = bytes;
    pinned_small_on_host_ = small_on_host;
  }

  // Device -> host copy of `bytes` (synchronous).  Large copies to
  // pageable memory go through pinned staging slots, emptied by several
  // host threads while the copy engine fills the next slot.
  void download(void* dst, const void* src, size_t bytes);

 private:
  int dev_;
  cudaStream_t s_ = nullptr;
  const char* pinned_src_ = nullptr;
  bool pinned_small_on_host_ = false;
  size_t pinned_len_ = 0;
  bool in_pinned(const void* p, size_t n) const {
    return pinned_src_ && (const char*)p >= pinned_src_ && (const char*)p + n <= pinned_src_ + pinned_len_;
  }
  std::unique_ptr<DeviceBuf> status_;   // dcf_status slots of a batch
  size_t status_cap_ = 0;
  std::unique_ptr<DeviceBuf> aux_;      // status word of uploads and scans outside a batch
  static constexpr int kSlots = 4;
  static constexpr size_t kSlotBytes = 16u << 20;
  void* pinned_[kSlots] = {nullptr};
  cudaEvent_t slot_ev_[kSlots] = {nullptr};
  void ensure_pinned();
  void hash_async(const std::vector<std::shared_ptr<DeviceBuf>>& bufs, const std::vector<DenseValue*>& vs,
                  std::unique_ptr<DeviceBuf>& desc, std::unique_ptr<DeviceBuf>& out);
  void upload_image(const std::vector<ImagePiece>& pcs, size_t total, char* arena);
  void download_image(const std::vector<ImagePiece>& pcs, size_t total);
  void run_batched(const std::vector<FoldRequest*>& reqs, const std::vector<const void*>& ls,
                   const std::vector<const void*>& rs, std::vector<std::shared_ptr<DeviceBuf>>& outs,
                   std::vector<dcf_status>& hst);
  void set_device();
  void check(int rc, const char* what);
  void sync();
  dcf_status* statuses(size_t n);
};

// Bare `canonicalize` over several GPUs.  Every fold that canonicalize
// runs element by element maps element i of its operands to element i of
// its result, so a large constant is cut into contiguous element ranges,
// range g living on GPU g, and each fold of such constants runs as one fold
// per range, on all GPUs at once.  Through a chain of folds the ranges stay
// aligned and no bytes cross GPUs; results come back to the host range by
// range.  Small constants (under kMinElements) stay whole on the first GPU.
//
// A sharded constant keeps its ranges in DenseValue::parts.  Its hash is a
// fixed combination of the ranges' hashes, so two constants of the same
// type compare equal exactly when their ranges do; an all-equal range that
// came back as one element hashes as its expansion.  The result of a fold
// is one element when every range came back as the same single element,
// which is when the kernel over the whole range would have said so.
class ShardedEngine : public Engine {
 public:
  explicit ShardedEngine(std::vector<Engine*> subs);
  static constexpr uint64_t kMinElements = 1u << 18;
  static constexpr uint64_t kAlign = 4096;  // range boundaries, in elements
  int device() const override { return subs_[0]->device(); }
  void execute(const std::vector<FoldRequest*>& reqs) override;
  void to_device(DenseValue& v) override;
  void to_device_all(const std::vector<DenseValue*>& vs) override;
  void to_host(DenseValue& v) override;
  void to_host_all(const std::vector<DenseValue*>& vs) override;
  std::string hex_of(DenseValue& v) override;
  uint64_t bits0_of(DenseValue& v) override;
  uint64_t hash_of(DenseValue& v) override;
  bool all_equal(DenseValue& v) override;

 private:
  std::vector<Engine*> subs_;
  bool shardable(const DenseValue& v) const;
  uint64_t chunk(uint64_t n) const;
  void split(DenseValue& v);
  Engine* owner(const DenseValue& v) const;
  uint64_t part_hash(const DenseValue& whole, size_t g);
  // Run f(g) for every range g on its own host thread.
  template <class F> void each(size_t parts, F&& f);
};

}  // namespace dco
