// conv_tc_kernel instantiations for the none epilogue activation (one unit per activation so the
// kernels compile in parallel).
#include "conv_tc_kernel.cuh"

namespace sdx {
template int launch_tc<ACT_NONE, 4, 4>(int, int, size_t, cudaStream_t, const CUtensorMap&, const CUtensorMap&,
                                    const CUtensorMap&, const CUtensorMap&, const TcArgs&);
template int launch_tc<ACT_NONE, 4, 2>(int, int, size_t, cudaStream_t, const CUtensorMap&, const CUtensorMap&,
                                    const CUtensorMap&, const CUtensorMap&, const TcArgs&);
template int launch_tc<ACT_NONE, 1, 4>(int, int, size_t, cudaStream_t, const CUtensorMap&, const CUtensorMap&,
                                    const CUtensorMap&, const CUtensorMap&, const TcArgs&);
template int launch_tc<ACT_NONE, 1, 2>(int, int, size_t, cudaStream_t, const CUtensorMap&, const CUtensorMap&,
                                    const CUtensorMap&, const CUtensorMap&, const TcArgs&);
template int launch_tc<ACT_NONE, 2, 2>(int, int, size_t, cudaStream_t, const CUtensorMap&, const CUtensorMap&,
                                    const CUtensorMap&, const CUtensorMap&, const TcArgs&);
template int launch_tc<ACT_NONE, 0, 4>(int, int, size_t, cudaStream_t, const CUtensorMap&, const CUtensorMap&,
                                    const CUtensorMap&, const CUtensorMap&, const TcArgs&);
template int launch_tc<ACT_NONE, 0, 2>(int, int, size_t, cudaStream_t, const CUtensorMap&, const CUtensorMap&,
                                    const CUtensorMap&, const CUtensorMap&, const TcArgs&);
// the fused CTC head (EPI = 5) has no activation
template int launch_tc<ACT_NONE, 5, 4>(int, int, size_t, cudaStream_t, const CUtensorMap&, const CUtensorMap&,
                                    const CUtensorMap&, const CUtensorMap&, const TcArgs&);
template int launch_tc<ACT_NONE, 5, 2>(int, int, size_t, cudaStream_t, const CUtensorMap&, const CUtensorMap&,
                                    const CUtensorMap&, const CUtensorMap&, const TcArgs&);
template int launch_tc<ACT_NONE, 6, 2>(int, int, size_t, cudaStream_t, const CUtensorMap&, const CUtensorMap&,
                                    const CUtensorMap&, const CUtensorMap&, const TcArgs&);
}  // namespace sdx
