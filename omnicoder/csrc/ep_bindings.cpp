// Tensor-level bindings of the expert-parallel exchange kernels (ep_comm.cu).
// Peer addresses arrive as Python ints (device pointers of peer-mapped
// symmetric memory, valid in this process) with the row capacity of each.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "ep_comm.h"

namespace omni {

namespace {
cudaStream_t stream() { return at::cuda::getCurrentCUDAStream().stream(); }

EpPeers make_peers(const std::vector<int64_t>& ptrs, const std::vector<int64_t>& rows) {
  TORCH_CHECK(ptrs.size() <= (size_t)kEpMaxRanks, "expert parallel: at most ", kEpMaxRanks, " ranks");
  TORCH_CHECK(rows.empty() || rows.size() == ptrs.size(), "expert parallel: rows per rank");
  EpPeers p;
  for (int i = 0; i < kEpMaxRanks; ++i) {
    p.ptr[i] = i < (int)ptrs.size() ? (unsigned long long)ptrs[i] : 0ull;
    p.rows[i] = (i < (int)rows.size()) ? (int)rows[i] : 0;
  }
  return p;
}

void check(const at::Tensor& t, at::ScalarType dt, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == dt && t.is_contiguous(), name, ": wrong device/dtype/layout");
}
}  // namespace

at::Tensor ep_dispatch_t(const at::Tensor& x, const at::Tensor& idx, const at::Tensor& pos, const at::Tensor& loc_off,
                         const at::Tensor& dst_base, const at::Tensor& keep_lim, const at::Tensor& wts,
                         const std::vector<int64_t>& x_ptrs, const std::vector<int64_t>& meta_ptrs,
                         const std::vector<int64_t>& rows, int64_t El, int64_t me) {
  check(x, at::kBFloat16, "x");
  check(idx, at::kInt, "idx");
  check(pos, at::kInt, "pos");
  check(wts, at::kFloat, "wts");
  const c10::cuda::CUDAGuard g(x.device());
  const int64_t T = idx.size(0), K = idx.size(1), D = x.size(1), E = dst_base.numel();
  TORCH_CHECK(D % 8 == 0, "ep_dispatch: D % 8");
  auto slot = at::empty({T, K}, idx.options());
  ep_dispatch(x.data_ptr(), idx.data_ptr<int>(), pos.data_ptr<int>(), loc_off.data_ptr<int>(),
              dst_base.data_ptr<int>(), keep_lim.data_ptr<int>(), wts.data_ptr<float>(), make_peers(x_ptrs, rows),
              make_peers(meta_ptrs, rows), slot.data_ptr<int>(), (int)T, (int)K, (int)E, (int)El, (int)D, (int)me,
              stream());
  return slot;
}

void ep_push_t(const at::Tensor& src, const at::Tensor& slot, const at::Tensor& idx, const std::vector<int64_t>& ptrs,
               const std::vector<int64_t>& rows, int64_t El) {
  check(src, at::kBFloat16, "src");
  const c10::cuda::CUDAGuard g(src.device());
  ep_push(src.data_ptr(), slot.data_ptr<int>(), idx.data_ptr<int>(), make_peers(ptrs, rows), (int)slot.size(0),
          (int)slot.size(1), (int)El, (int)src.size(1), stream());
}

// out[t] = add[t] + sum_k w[t,k] ys[t*K+k] over kept pairs: the combine after the owners pushed their
// rows into this rank's slots ys [T*K, D] (local reads).
at::Tensor ep_combine_local_t(const at::Tensor& slot, const at::Tensor& ys, const c10::optional<at::Tensor>& w,
                              const c10::optional<at::Tensor>& add) {
  check(slot, at::kInt, "slot");
  check(ys, at::kBFloat16, "ys");
  const c10::cuda::CUDAGuard g(slot.device());
  const int64_t T = slot.size(0), K = slot.size(1), D = ys.size(1);
  TORCH_CHECK(K <= 16 && ys.size(0) == T * K && D % 8 == 0, "ep_combine_local: ys [T*K, D], top-k <= 16");
  auto out = at::empty({T, D}, ys.options());
  if (add.has_value()) check(*add, at::kBFloat16, "add");
  if (w.has_value()) check(*w, at::kFloat, "w");
  ep_combine(slot.data_ptr<int>(), slot.data_ptr<int>(), w.has_value() ? w->data_ptr<float>() : nullptr, EpPeers{},
             add.has_value() ? add->data_ptr() : nullptr, out.data_ptr(), (int)T, (int)K, 1, (int)D, stream(),
             ys.data_ptr());
  return out;
}

void ep_return_rows_t(const at::Tensor& y, const at::Tensor& meta, const at::Tensor& offsets,
                      const std::vector<int64_t>& ys_ptrs, const std::vector<int64_t>& ys_rows) {
  check(y, at::kBFloat16, "y");
  check(meta, at::kInt, "meta");
  check(offsets, at::kInt, "offsets");
  const c10::cuda::CUDAGuard g(y.device());
  TORCH_CHECK(meta.dim() == 2 && meta.size(1) == 4 && meta.size(0) >= y.size(0) && y.size(1) % 8 == 0,
              "ep_return_rows: meta [rows, 4], D % 8");
  ep_return_rows(y.data_ptr(), meta.data_ptr(), offsets.data_ptr<int>(), (int)offsets.numel() - 1,
                 make_peers(ys_ptrs, ys_rows), (int)y.size(0), (int)y.size(1), stream());
}

void ep_source_bwd_t(const at::Tensor& dout, const at::Tensor& ys, const at::Tensor& slot, const at::Tensor& idx,
                     const at::Tensor& w, at::Tensor& dwts, const std::vector<int64_t>& dy_ptrs,
                     const std::vector<int64_t>& rows, int64_t El) {
  check(dout, at::kBFloat16, "dout");
  check(ys, at::kBFloat16, "ys");
  check(slot, at::kInt, "slot");
  check(idx, at::kInt, "idx");
  check(w, at::kFloat, "w");
  check(dwts, at::kFloat, "dwts");
  const c10::cuda::CUDAGuard g(dout.device());
  const int64_t T = slot.size(0), K = slot.size(1), D = dout.size(1);
  TORCH_CHECK(ys.size(0) == T * K && ys.size(1) == D && D % 8 == 0 && dwts.numel() == T * K,
              "ep_source_bwd: shapes");
  ep_source_bwd(dout.data_ptr(), ys.data_ptr(), slot.data_ptr<int>(), idx.data_ptr<int>(), w.data_ptr<float>(),
                dwts.data_ptr<float>(), make_peers(dy_ptrs, rows), (int)T, (int)K, (int)El, (int)D, stream());
}

at::Tensor ep_combine_t(const at::Tensor& slot, const at::Tensor& idx, const c10::optional<at::Tensor>& w,
                        const std::vector<int64_t>& ptrs, const std::vector<int64_t>& rows, int64_t El, int64_t D,
                        const c10::optional<at::Tensor>& add) {
  check(slot, at::kInt, "slot");
  const c10::cuda::CUDAGuard g(slot.device());
  const int64_t T = slot.size(0), K = slot.size(1);
  TORCH_CHECK(K <= 16, "ep_combine: top-k <= 16");
  auto out = at::empty({T, D}, slot.options().dtype(at::kBFloat16));
  if (add.has_value()) check(*add, at::kBFloat16, "add");
  if (w.has_value()) check(*w, at::kFloat, "w");
  ep_combine(slot.data_ptr<int>(), idx.data_ptr<int>(), w.has_value() ? w->data_ptr<float>() : nullptr,
             make_peers(ptrs, rows), add.has_value() ? add->data_ptr() : nullptr, out.data_ptr(), (int)T, (int)K,
             (int)El, (int)D, stream());
  return out;
}

void ep_owner_bwd_t(at::Tensor& dy, const at::Tensor& y, const at::Tensor& meta, const at::Tensor& offsets,
                    const at::Tensor& kept, const std::vector<int64_t>& dw_ptrs, const std::vector<int64_t>& dw_rows) {
  check(dy, at::kBFloat16, "dy");
  check(y, at::kBFloat16, "y");
  const c10::cuda::CUDAGuard g(dy.device());
  const int64_t El = kept.numel();
  TORCH_CHECK(El <= kEpMaxRanks * 32, "ep_owner_bwd: too many local experts");
  ep_owner_bwd(dy.data_ptr(), y.data_ptr(), meta.data_ptr(), offsets.data_ptr<int>(), kept.data_ptr<int>(), (int)El,
               make_peers(dw_ptrs, dw_rows), (int)dy.size(0), (int)dy.size(1), stream());
}

void ep_pad_rows_t(at::Tensor& x, const c10::optional<at::Tensor>& meta, const at::Tensor& offsets,
                   const at::Tensor& kept) {
  check(x, at::kBFloat16, "x");
  const c10::cuda::CUDAGuard g(x.device());
  ep_pad_rows(x.data_ptr(), meta.has_value() ? meta->data_ptr() : nullptr, offsets.data_ptr<int>(),
              kept.data_ptr<int>(), (int)kept.numel(), (int)x.size(0), (int)x.size(1), stream());
}

void ep_barrier_t(const std::vector<int64_t>& sig_ptrs, int64_t me, int64_t epoch, int64_t device) {
  const c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  ep_barrier(make_peers(sig_ptrs, {}), (int)me, (int)sig_ptrs.size(), (unsigned)(epoch & 0xffffffffll), stream());
}

void ep_barrier_dev_t(const std::vector<int64_t>& sig_ptrs, int64_t me, at::Tensor& epoch_ctr) {
  check(epoch_ctr, at::kInt, "epoch_ctr");
  const c10::cuda::CUDAGuard g(epoch_ctr.device());
  ep_barrier_dev(make_peers(sig_ptrs, {}), (int)me, (int)sig_ptrs.size(),
                 reinterpret_cast<unsigned*>(epoch_ctr.data_ptr<int>()), stream());
}

// -> (dst_base [E], keep_lim [E], offs_local [El + 1], kept_local [El]) written into the given tensors
void ep_exchange_layout_t(const at::Tensor& counts, const std::vector<int64_t>& board_ptrs,
                          const std::vector<int64_t>& sig_ptrs, int64_t me, at::Tensor& epoch_ctr, int64_t El,
                          int64_t capacity, int64_t seg_cap, at::Tensor& dst_base, at::Tensor& keep_lim,
                          at::Tensor& offs_local, at::Tensor& kept_local, at::Tensor& dropped,
                          const c10::optional<at::Tensor>& src_pref) {
  for (const at::Tensor* t : std::initializer_list<const at::Tensor*>{&counts, &epoch_ctr, &dst_base, &keep_lim,
                                                                       &offs_local, &kept_local, &dropped})
    check(*t, at::kInt, "ep_exchange_layout");
  const int64_t E = counts.numel();
  const int64_t n = (int64_t)board_ptrs.size();
  TORCH_CHECK(E >= 1 && E <= 1024 && El >= 1 && E % El == 0 && E / El == n, "ep_exchange_layout: E = El * ranks");
  TORCH_CHECK(sig_ptrs.size() == board_ptrs.size(), "ep_exchange_layout: one signal area per rank");
  TORCH_CHECK(dst_base.numel() == E && keep_lim.numel() == E && offs_local.numel() == El + 1 &&
                  kept_local.numel() == El && dropped.numel() >= 1,
              "ep_exchange_layout: output sizes");
  TORCH_CHECK(seg_cap > 0 && seg_cap % 128 == 0, "ep_exchange_layout: seg_cap must be a positive multiple of 128");
  if (src_pref.has_value()) {
    check(*src_pref, at::kInt, "ep_exchange_layout src_pref");
    TORCH_CHECK(src_pref->numel() == El * (n + 1), "ep_exchange_layout: src_pref [El, ranks + 1]");
  }
  const c10::cuda::CUDAGuard g(counts.device());
  ep_exchange_layout(make_peers(board_ptrs, {}), make_peers(sig_ptrs, {}), (int)me, (int)n,
                     reinterpret_cast<unsigned*>(epoch_ctr.data_ptr<int>()), counts.data_ptr<int>(), (int)E, (int)El,
                     (int)capacity, (int)seg_cap, dst_base.data_ptr<int>(), keep_lim.data_ptr<int>(),
                     offs_local.data_ptr<int>(), kept_local.data_ptr<int>(), dropped.data_ptr<int>(), stream(),
                     src_pref.has_value() ? src_pref->data_ptr<int>() : nullptr);
}

void ep_signal_t(const std::vector<int64_t>& flag_ptrs, int64_t me, at::Tensor& sig_ctr) {
  check(sig_ctr, at::kInt, "ep_signal");
  const c10::cuda::CUDAGuard g(sig_ctr.device());
  TORCH_CHECK(!flag_ptrs.empty() && flag_ptrs.size() <= (size_t)kEpMaxRanks, "ep_signal: 1..8 ranks");
  ep_signal(make_peers(flag_ptrs, {}), (int)me, (int)flag_ptrs.size(),
            reinterpret_cast<unsigned*>(sig_ctr.data_ptr<int>()), stream());
}

void zero_rs_t(const std::vector<int64_t>& g_ptrs, int64_t lo, int64_t n, double scale, at::Tensor& out,
               const c10::optional<at::Tensor>& norm_sq) {
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kFloat && out.is_contiguous() && out.numel() >= n,
              "zero_rs: fp32 shard output");
  TORCH_CHECK(lo % 8 == 0, "zero_rs: shard offset must be a multiple of 8 elements");
  const c10::cuda::CUDAGuard gd(out.device());
  zero_rs(make_peers(g_ptrs, {}), (int)g_ptrs.size(), lo, n, (float)scale, out.data_ptr<float>(),
          norm_sq.has_value() ? norm_sq->data_ptr<float>() : nullptr, stream());
}

void zero_adamw_push_t(at::Tensor& p, at::Tensor& m, at::Tensor& v, const at::Tensor& g,
                       const std::vector<int64_t>& dst_ptrs, int64_t lo, double lr, double b1, double b2, double eps,
                       double wd, int64_t step, const c10::optional<at::Tensor>& norm_sq, double max_norm) {
  for (const at::Tensor* t : std::initializer_list<const at::Tensor*>{&p, &m, &v, &g})
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kFloat && t->is_contiguous() && t->numel() == p.numel(),
                "zero_adamw_push: fp32 master / moments / gradient shards of one size");
  TORCH_CHECK(lo % 8 == 0, "zero_adamw_push: shard offset must be a multiple of 8 elements");
  const c10::cuda::CUDAGuard gd(p.device());
  zero_adamw_push(p.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(), g.data_ptr<float>(),
                  make_peers(dst_ptrs, {}), (int)dst_ptrs.size(), lo, p.numel(), (float)lr, (float)b1, (float)b2,
                  (float)eps, (float)wd, (int)step, norm_sq.has_value() ? norm_sq->data_ptr<float>() : nullptr,
                  (float)max_norm, stream());
}

void register_ep(pybind11::module_& m) {
  m.def("ep_dispatch", &ep_dispatch_t);
  m.def("ep_push", &ep_push_t);
  m.def("ep_combine", &ep_combine_t);
  m.def("ep_combine_local", &ep_combine_local_t);
  m.def("ep_source_bwd", &ep_source_bwd_t);
  m.def("ep_return_rows", &ep_return_rows_t);
  m.def("ep_owner_bwd", &ep_owner_bwd_t);
  m.def("ep_pad_rows", &ep_pad_rows_t);
  m.def("ep_barrier", &ep_barrier_t);
  m.def("ep_barrier_dev", &ep_barrier_dev_t);
  m.def("ep_exchange_layout", &ep_exchange_layout_t, py::arg("counts"), py::arg("board_ptrs"), py::arg("sig_ptrs"),
        py::arg("me"), py::arg("epoch_ctr"), py::arg("El"), py::arg("capacity"), py::arg("seg_cap"),
        py::arg("dst_base"), py::arg("keep_lim"), py::arg("offs_local"), py::arg("kept_local"), py::arg("dropped"),
        py::arg("src_pref") = py::none());
  m.def("ep_signal", &ep_signal_t);
  m.def("zero_rs", &zero_rs_t, py::arg("g_ptrs"), py::arg("lo"), py::arg("n"), py::arg("scale"), py::arg("out"),
        py::arg("norm_sq") = py::none());
  m.def("zero_adamw_push", &zero_adamw_push_t, py::arg("p"), py::arg("m"), py::arg("v"), py::arg("g"),
        py::arg("dst_ptrs"), py::arg("lo"), py::arg("lr"), py::arg("b1"), py::arg("b2"), py::arg("eps"), py::arg("wd"),
        py::arg("step"), py::arg("norm_sq") = py::none(), py::arg("max_norm") = 0.0);
}

}  // namespace omni
