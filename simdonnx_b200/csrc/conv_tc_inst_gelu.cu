// conv_tc_kernel instantiations for the gelu epilogue activation (one unit per activation so the
// kernels compile in parallel).
#include "conv_tc_kernel.cuh"

namespace sdx {
template int launch_tc<ACT_GELU, 4, 4>(int, int, size_t, cudaStream_t, const CUtensorMap&, const CUtensorMap&,
                                    const CUtensorMap&, const CUtensorMap&, const TcArgs&);
template int launch_tc<ACT_GELU, 4, 2>(int, int, size_t, cudaStream_t, const CUtensorMap&, const CUtensorMap&,
                                    const CUtensorMap&, const CUtensorMap&, const TcArgs&);
template int launch_tc<ACT_GELU, 1, 4>(int, int, size_t, cudaStream_t, const CUtensorMap&, const CUtensorMap&,
                                    const CUtensorMap&, const CUtensorMap&, const TcArgs&);
template int launch_tc<ACT_GELU, 1, 2>(int, int, size_t, cudaStream_t, const CUtensorMap&, const CUtensorMap&,
                                    const CUtensorMap&, const CUtensorMap&, const TcArgs&);
template int launch_tc<ACT_GELU, 2, 2>(int, int, size_t, cudaStream_t, const CUtensorMap&, const CUtensorMap&,
                                    const CUtensorMap&, const CUtensorMap&, const TcArgs&);
template int launch_tc<ACT_GELU, 0, 4>(int, int, size_t, cudaStream_t, const CUtensorMap&, const CUtensorMap&,
                                    const CUtensorMap&, const CUtensorMap&, const TcArgs&);
template int launch_tc<ACT_GELU, 0, 2>(int, int, size_t, cudaStream_t, const CUtensorMap&, const CUtensorMap&,
                                    const CUtensorMap&, const CUtensorMap&, const TcArgs&);
template int launch_tc<ACT_GELU, 6, 2>(int, int, size_t, cudaStream_t, const CUtensorMap&, const CUtensorMap&,
                                    const CUtensorMap&, const CUtensorMap&, const TcArgs&);
}  // namespace sdx
