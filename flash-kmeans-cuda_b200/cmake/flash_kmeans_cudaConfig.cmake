# CMake package of the prebuilt flash_kmeans_cuda B200 libraries (built by
# flash-kmeans-cuda_b200/build.py). Same package and target names as the
# reference's installed package (flash_kmeans_cuda/CMakeLists.txt:100-125,
# cmake/flash_kmeans_cudaConfig.cmake.in), so C++ consumers keep
#
#   find_package(flash_kmeans_cuda CONFIG REQUIRED)
#   target_link_libraries(app PRIVATE flash_kmeans_cuda::flash_kmeans_cuda)
#
# with CMAKE_PREFIX_PATH (or flash_kmeans_cuda_DIR) pointing at this folder.
#
# Targets:
#   flash_kmeans_cuda::fkc_capi           C-ABI only (include/fkc_capi.h), no torch
#   flash_kmeans_cuda::flash_kmeans_cuda  libtorch fkc:: API
#                                         (include/flash_kmeans_cuda/flash_kmeans_cuda.h);
#                                         defined when Torch is found, as in the reference.

get_filename_component(_fkc_pkg "${CMAKE_CURRENT_LIST_DIR}/.." ABSOLUTE)
get_filename_component(_fkc_root "${_fkc_pkg}/.." ABSOLUTE)
set(_fkc_libdir "${_fkc_pkg}/flash_kmeans_cuda")

if(NOT EXISTS "${_fkc_libdir}/libfkc_b200.so")
  set(flash_kmeans_cuda_FOUND FALSE)
  set(flash_kmeans_cuda_NOT_FOUND_MESSAGE
      "libfkc_b200.so not built: run python flash-kmeans-cuda_b200/build.py")
  return()
endif()

include(CMakeFindDependencyMacro)
find_dependency(CUDAToolkit)

if(NOT TARGET flash_kmeans_cuda::fkc_capi)
  add_library(flash_kmeans_cuda::fkc_capi SHARED IMPORTED)
  set_target_properties(flash_kmeans_cuda::fkc_capi PROPERTIES
    IMPORTED_LOCATION "${_fkc_libdir}/libfkc_b200.so"
    IMPORTED_SONAME "libfkc_b200.so"
    INTERFACE_INCLUDE_DIRECTORIES "${_fkc_root}/include"
    INTERFACE_LINK_LIBRARIES "CUDA::cudart")
endif()

find_package(Torch QUIET)
if(Torch_FOUND AND EXISTS "${_fkc_libdir}/libflash_kmeans_cuda.so"
   AND NOT TARGET flash_kmeans_cuda::flash_kmeans_cuda)
  add_library(flash_kmeans_cuda::flash_kmeans_cuda SHARED IMPORTED)
  set_target_properties(flash_kmeans_cuda::flash_kmeans_cuda PROPERTIES
    IMPORTED_LOCATION "${_fkc_libdir}/libflash_kmeans_cuda.so"
    IMPORTED_SONAME "libflash_kmeans_cuda.so"
    INTERFACE_INCLUDE_DIRECTORIES "${_fkc_root}/include;${TORCH_INCLUDE_DIRS}"
    INTERFACE_LINK_LIBRARIES "flash_kmeans_cuda::fkc_capi;${TORCH_LIBRARIES};CUDA::cudart")
endif()

set(flash_kmeans_cuda_VERSION "0.1.0")
unset(_fkc_pkg)
unset(_fkc_root)
unset(_fkc_libdir)
