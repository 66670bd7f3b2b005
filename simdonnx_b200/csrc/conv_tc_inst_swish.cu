// conv_tc_kernel instantiations for the swish epilogue activation (one unit per activation so the
// kernels compile in parallel).
#include "conv_tc_kernel.cuh"

namespace sdx {
template int launch_tc<ACT_SWISH, 4, 4>(int, int, size_t, cudaStream_t, const CUtensorMap&, const CUtensorMap&,
                                    const CUtensorMap&, const CUtensorMap&, const TcArgs&);
template int launch_tc<ACT_SWISH, 4, 2>(int, int, size_t, cudaStream_t, const CUtensorMap&, const CUtensorMap&,
                                    const CUtensorMap&, const CUtensorMap&, const TcArgs&);
template int launch_tc<ACT_SWISH, 1, 4>(int, int, size_t, cudaStream_t, const CUtensorMap&, const CUtensorMap&,
                                    const CUtensorMap&, const CUtensorMap&, const TcArgs&);
template int launch_tc<ACT_SWISH, 1, 2>(int, int, size_t, cudaStream_t, const CUtensorMap&, const CUtensorMap&,
                                    const CUtensorMap&, const CUtensorMap&, const TcArgs&);
template int launch_tc<ACT_SWISH, 2, 2>(int, int, size_t, cudaStream_t, const CUtensorMap&, const CUtensorMap&,
                                    const CUtensorMap&, const CUtensorMap&, const TcArgs&);
template int launch_tc<ACT_SWISH, 0, 4>(int, int, size_t, cudaStream_t, const CUtensorMap&, const CUtensorMap&,
                                    const CUtensorMap&, const CUtensorMap&, const TcArgs&);
template int launch_tc<ACT_SWISH, 0, 2>(int, int, size_t, cudaStream_t, const CUtensorMap&, const CUtensorMap&,
                                    const CUtensorMap&, const CUtensorMap&, const TcArgs&);
template int launch_tc<ACT_SWISH, 6, 2>(int, int, size_t, cudaStream_t, const CUtensorMap&, const CUtensorMap&,
                                    const CUtensorMap&, const CUtensorMap&, const TcArgs&);
}  // namespace sdx
