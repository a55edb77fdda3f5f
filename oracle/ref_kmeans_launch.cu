// Host launchers for the reference's two k-means kernels, which the
// reference declares (csrc/clustering/kmeans.cpp:8-18) but never defines.
// Test infrastructure: linked (relocatable device code) against the
// unmodified csrc/kernels/kmeans.cu by oracle/build_ref.sh, so golden k-means
// vectors come from the reference's own device code.  Launch shapes follow the
// kernels' comments: one thread per point (kmeans.cu:19), one block per
// centroid with d floats of dynamic shared memory (kmeans.cu:58-61).
#include <cuda_runtime.h>

namespace rapidadb {
__global__ void assign_clusters_kernel(const float* points, const float* centroids,
                                       int* assignments, float* distances, int n, int k, int d);
__global__ void update_centroids_kernel(const float* points, const int* assignments,
                                        float* new_centroids, int* counts, int n, int k, int d);
}  // namespace rapidadb

extern "C" int ref_kmeans_assign(const float* points, const float* centroids, int* assignments,
                                 float* distances, int n, int k, int d) {
    if (n <= 0) return 0;
    rapidadb::assign_clusters_kernel<<<(n + 255) / 256, 256>>>(points, centroids, assignments,
                                                                distances, n, k, d);
    return (int)cudaDeviceSynchronize();
}

// new_centroids must hold the previous centroids on entry: the reference
// leaves a centroid with no points unwritten.
extern "C" int ref_kmeans_update(const float* points, const int* assignments,
                                 float* new_centroids, int* counts, int n, int k, int d) {
    if (k <= 0) return 0;
    cudaError_t e = cudaMemset(counts, 0, sizeof(int) * (size_t)k);
    if (e != cudaSuccess) return (int)e;
    rapidadb::update_centroids_kernel<<<k, 256, sizeof(float) * (size_t)d>>>(
        points, assignments, new_centroids, counts, n, k, d);
    return (int)cudaDeviceSynchronize();
}
