// pybind11 module over the reference's libtorch API (flash_kmeans_cuda/csrc/
// flash_kmeans_cuda.h:34-75), so tests can run the reference's own CUDA kernels
// on the GPU beside this library's. Test infrastructure only; built by
// oracle/build_ref.sh into oracle/_ref/.
#include <torch/extension.h>

#include "flash_kmeans_cuda.h"

PYBIND11_MODULE(fkc_ref_shim, m) {
  m.doc() = "reference flash-kmeans-cuda fkc:: API (comparator)";
  m.def("euclid_assign", &fkc::euclid_assign, "reference assign (allocates ids)");
  m.def("euclid_assign_out", &fkc::euclid_assign_out, "reference assign into ids");
  m.def("centroid_update_sorted", &fkc::centroid_update_sorted,
        "reference sorted-run accumulate (zeroes sums/counts first)");
  m.def("centroid_update_sorted_indexed", &fkc::centroid_update_sorted_indexed,
        "reference indexed sorted-run accumulate (zeroes sums/counts first)");
  m.def("centroid_finalize_out", &fkc::centroid_finalize_out, "reference finalize into out");
}
